import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200, sm_100a) device")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this process")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def pytest_sessionstart(session):
    """Build libcuopx.so (and the oracle) when missing or stale — a no-op on
    an up-to-date tree — so a fresh checkout runs the suite directly."""
    import shutil
    import subprocess

    from cuop_b200 import build

    if shutil.which("nvcc") or os.path.exists("/usr/local/cuda/bin/nvcc"):
        build.build()
    if not (ROOT / "oracle" / "liboracle.so").exists():
        subprocess.run(["make", "-s", "-C", str(ROOT / "oracle"), "all"], check=True)


@pytest.fixture(scope="session", autouse=True)
def _builtin_gemm_selection():
    """Kernel-parity tests name the kernel each shape must reach under the
    built-in selection; the shipped tuning table is cleared for the session
    (tests of the table load their own)."""
    from cuop_b200 import _native as N

    N.lib().cuopx_tuning_clear()
    yield


@pytest.fixture(scope="session")
def dev():
    import torch

    return torch.device("cuda", 0)


@pytest.fixture(autouse=True)
def _no_device_error(request):
    """Every GPU test must leave the device error word clean."""
    yield
    if "gpu" in request.keywords:
        import cuop_b200 as cx

        code = cx.device_error()
        if code:
            cx.clear_device_error()
        assert code == 0, f"device-side error word set: {code}"


@pytest.fixture
def fp32_ffma():
    """Run a test with fp32 GEMM forced onto the FFMA kernels (bit-reproducible
    ascending-k order); restores the default mode afterwards."""
    from cuop_b200 import _native as N

    assert N.lib().cuopx_set_fp32_gemm_mode(N.FP32_FFMA) == 0
    yield
    assert N.lib().cuopx_set_fp32_gemm_mode(N.FP32_AUTO) == 0
