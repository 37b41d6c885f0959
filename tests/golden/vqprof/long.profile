VQPROF 1
artifact bfdfd4c2eb92acd6
gpu NVIDIA B200
gemv 4 4096 64 2560 1 3 512                                                                                                                                                                                                                                                                                                                                                                                                                                                                                                                                                                                                                        gemv 4 4096 96 2560 1 4 512 7.0
prefill 4 4096 64 2560 1 2 128 64
