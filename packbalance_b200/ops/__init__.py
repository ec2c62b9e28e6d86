"""Autograd-aware ops.  CUDA tensors run the native sm_100a kernels (and fail loudly
if the extension is missing); CPU tensors run the PyTorch reference math."""
