"""sm_100a kernels with their fp32 PyTorch oracles."""
