VQPROF 1
artifact bfdfd4c2eb92acd6
gpu NVIDIA B200 xxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxxx  
driver 12090 
gemv 4 256 8 64 1 1 128 10.0
prefill 4 256 32 256 1 1 64 64
