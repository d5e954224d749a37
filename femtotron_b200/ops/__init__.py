"""Kernel entry points (sm_100a on CUDA tensors, PyTorch math on CPU tensors)."""
from .ext import check_kernel_errors, has_native, native, KernelTimeoutError
from .matmul import gemm, linear_dgrad, linear_fwd, linear_wgrad
from . import kernels, functional

__all__ = ["native", "has_native", "check_kernel_errors", "KernelTimeoutError", "gemm",
           "linear_fwd", "linear_dgrad", "linear_wgrad", "kernels", "functional"]
