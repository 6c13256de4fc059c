"""Model zoo built on the sm_100a kernels."""
