"""Hand-written sm_100a kernels behind torch-shaped functions.

Each op runs its CUDA kernel for CUDA tensors (bf16) and an FP32 torch computation for
CPU tensors; there is no other path.
"""

from . import _ext  # noqa: F401
from .gemm import KernelError, check_device_errors, linear, linear_dgrad, linear_wgrad  # noqa: F401
