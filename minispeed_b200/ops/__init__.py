"""sm_100a kernels (``minispeed_b200._C``) and their PyTorch-facing wrappers."""
