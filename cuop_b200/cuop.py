"""The reference's Python package surface (python/cuop/__init__.py) for the
BLAS operators, on the sm_100a kernels: `from cuop_b200 import cuop`, then
`cuop.tensor(...)`, `cuop.GemmFloat()`, `cuop.JITGemmFloat(gemm)`, ... as in
the reference's examples.  The classes come from the pybind11 module
`cuop_b200.core` (built over the C++ facade); the aliases and helpers follow
the reference package.  Operators outside the BLAS path are not provided.
"""
from __future__ import annotations

from .core import (  # noqa: F401
    AxpyDouble, AxpyFloat, BatchMatMulDouble, BatchMatMulFloat, CopyDouble, CopyFloat, DotDouble, DotFloat,
    GemmDouble, GemmFloat, GemvDouble, GemvFloat, GlobalJITConfig, JITConfig, JITGemmFloat, JITGemvFloat,
    MatMulDouble, MatMulFloat, PerformanceProfile, ScalDouble, ScalFloat, TensorDouble, TensorFloat, empty_cache,
    get_device, get_device_count, get_memory_info, ones, randn, set_device, synchronize, tensor, zeros,
)

Tensor = TensorFloat
Scal = ScalFloat
Axpy = AxpyFloat
Copy = CopyFloat
Dot = DotFloat
Gemm = GemmFloat
Gemv = GemvFloat
MatMul = MatMulFloat
BatchMatMul = BatchMatMulFloat
JITGemm = JITGemmFloat
JITGemv = JITGemvFloat


def is_cuda_available() -> bool:
    try:
        return get_device_count() > 0
    except Exception:
        return False


def get_default_jit_config() -> JITConfig:
    """The reference's default JIT configuration (the kernels here are
    ahead-of-time; the fields are kept for callers that set them)."""
    c = JITConfig()
    c.enable_jit = True
    c.kernel_type = "tiled"
    c.tile_size = 32
    c.block_size = 256
    c.optimization_level = "O2"
    c.enable_tensor_core = True
    c.enable_tma = True
    c.max_registers = 255
    c.enable_shared_memory_opt = True
    c.enable_loop_unroll = True
    c.enable_memory_coalescing = True
    return c


def get_default_global_jit_config() -> GlobalJITConfig:
    return GlobalJITConfig()
