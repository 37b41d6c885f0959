VQPROF 2
artifact bfdfd4c2eb92acd6
gpu NVIDIA B200
gemv 4 256 8 64 1 0 256 1.0
