VQPROF 1
artifact bfdfd4c2eb92acd6
gpu NVIDIA B200
driver 12090
gemv 4 4096 10240 2560 1 4 512 1346.2
gemv 4 4096 2560 4096 1 3 512
prefill 4 4096 6144 2560 1 2 128 64 5120.0
tune-note ignored by the reader
gemv 4 4096 10240 2560 1 3 256 900.0
