"""cuop_b200 — B200-native (sm_100a) dense BLAS hot path of cuOP.

The compute lives in libcuopx.so (hand-written CUDA for sm_100a behind the C
ABI in include/cuopx.h); this package is the Python host side over that ABI.
"""
from ._native import CuopError, lib, lib_path  # noqa: F401
from .ops import (  # noqa: F401
    asum, axpy, batched_gemm, batched_gemm_host, clear_device_error, copy, device_error, dot, gather_column_blocks,
    gemm, gemv, iamax, iamin, last_kernel, launch_count, nrm2, rot, scal, swap,
)

__version__ = "0.1.0"
