"""The pybind11 module `cuop_b200.core` builds and imports without a GPU and
exposes the reference's Python class names (python/cuop/core.cpp) for the
BLAS path."""
import pytest


def test_core_module_surface():
    from cuop_b200 import build

    build.build()  # no-op when libcuopx.so and the module are current
    from cuop_b200 import cuop, core

    for name in ("TensorFloat", "TensorDouble", "GemmFloat", "GemmDouble", "GemvFloat", "GemvDouble",
                 "MatMulFloat", "BatchMatMulFloat", "DotFloat", "AxpyFloat", "ScalFloat", "CopyFloat",
                 "JITGemmFloat", "JITGemvFloat", "JITConfig", "GlobalJITConfig", "PerformanceProfile",
                 "tensor", "zeros", "ones", "get_device_count", "synchronize", "get_memory_info"):
        assert hasattr(core, name), name
    assert cuop.Gemm is core.GemmFloat and cuop.Tensor is core.TensorFloat
    c = cuop.get_default_jit_config()
    assert (c.kernel_type, c.tile_size, c.block_size, c.optimization_level) == ("tiled", 32, 256, "O2")
    assert "kernel_type='tiled'" in repr(c)
    g = cuop.get_default_global_jit_config()
    assert g.enable_jit and g.cache_dir


def test_core_module_without_gpu_reports_no_device():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from cuop_b200 import cuop

    assert cuop.get_device_count() == 0 and not cuop.is_cuda_available()
