"""CPU tests of the C ABI: the library loads, exports exactly what
include/cuopx.h declares, and rejects bad arguments before touching a GPU."""
import ctypes as C
import re
from pathlib import Path

import pytest

import cuop_b200 as cx
from cuop_b200 import _native as N

ROOT = Path(__file__).resolve().parent.parent


def declared_symbols():
    text = (ROOT / "include" / "cuopx.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(cuopx_\w+)\s*\(", text)))


def test_library_loads_from_tree():
    L = cx.lib()
    assert Path(L._name).resolve() == (ROOT / "cuop_b200" / "libcuopx.so").resolve()
    assert L.cuopx_version() == 100


def test_every_declared_symbol_is_exported_and_bound():
    L = cx.lib()
    decl = declared_symbols()
    assert len(decl) >= 20
    bound = {name for name, _, _ in N.SIGNATURES}
    assert set(decl) == bound, set(decl) ^ bound
    for name in decl:
        assert hasattr(L, name), name


def test_status_codes_match_reference_enum():
    # include/util/status_code.hpp:28-161 of the reference
    assert (N.SUCCESS, N.NOT_IMPLEMENTED, N.TIMEOUT, N.CUDA_ERROR, N.OUT_OF_MEMORY) == (0, 1001, 1003, 2000, 3001)
    assert (N.INVALID_ARGUMENT, N.EXECUTION_TIMEOUT, N.KERNEL_NOT_FOUND, N.NOT_COMPILED) == (4001, 6002, 6005, 7003)
    assert (N.SHAPE_MISMATCH, N.UNSUPPORTED_TYPE) == (10002, 11001)


def test_header_status_macros_agree():
    text = (ROOT / "include" / "cuopx.h").read_text()
    macros = dict(re.findall(r"#define CUOPX_(\w+) (\d+)", text))
    for name in ("SUCCESS", "CUDA_ERROR", "INVALID_ARGUMENT", "SHAPE_MISMATCH", "UNSUPPORTED_TYPE"):
        assert int(macros[name]) == getattr(N, name)


def test_argument_validation_without_gpu():
    L = cx.lib()
    # negative sizes
    assert L.cuopx_gemm(N.F32, 0, 0, -1, 4, 4, 1.0, 16, 4, 16, 4, 0.0, 16, 4, None) == N.INVALID_ARGUMENT
    # unknown dtype
    assert L.cuopx_gemm(99, 0, 0, 4, 4, 4, 1.0, 16, 4, 16, 4, 0.0, 16, 4, None) == N.UNSUPPORTED_TYPE
    # empty problems are no-ops
    assert L.cuopx_gemm(N.F32, 0, 0, 0, 4, 4, 1.0, None, 4, None, 4, 0.0, None, 4, None) == N.SUCCESS
    assert L.cuopx_gemv(N.F32, 0, 0, 5, 1.0, None, 5, None, 0.0, None, None, 0, None) == N.SUCCESS
    # null operands with real sizes
    assert L.cuopx_gemm(N.F32, 0, 0, 4, 4, 4, 1.0, None, 4, 16, 4, 0.0, 64, 4, None) == N.INVALID_ARGUMENT
    # leading dimension too small
    assert L.cuopx_gemm(N.F32, 0, 0, 4, 4, 8, 1.0, 4096, 4, 8192, 4, 0.0, 16384, 4, None) == N.INVALID_ARGUMENT
    # transposed A needs lda >= M
    assert L.cuopx_gemm(N.F32, 1, 0, 8, 4, 4, 1.0, 4096, 4, 8192, 4, 0.0, 16384, 4, None) == N.INVALID_ARGUMENT
    # C overlapping A
    assert L.cuopx_gemm(N.F32, 0, 0, 4, 4, 4, 1.0, 4096, 4, 8192, 4, 0.0, 4096 + 16, 4, None) == N.INVALID_ARGUMENT
    # gemv: lda < N, y overlapping x
    assert L.cuopx_gemv(N.F32, 0, 4, 8, 1.0, 4096, 4, 8192, 0.0, 16384, None, 0, None) == N.INVALID_ARGUMENT
    assert L.cuopx_gemv(N.F32, 0, 4, 4, 1.0, 4096, 4, 8192, 0.0, 8192, None, 0, None) == N.INVALID_ARGUMENT
    # the allocation-free GEMV runs the same checks before it sizes its scratch: the bf16
    # transposed 8191 x 8192 shape (whose kernel would need more than its scratch) with
    # lda < M is an invalid argument, not a resource shortage; and a null y as well
    M, Nn = 8191, 8192
    A, x, y = 1 << 32, 2 << 32, 3 << 32  # far apart, never dereferenced
    assert L.cuopx_gemv_noalloc(N.BF16, 1, M, Nn, 1.0, A, M - 1, x, 0.0, y, None) == N.INVALID_ARGUMENT
    assert L.cuopx_gemv_noalloc(N.BF16, 1, M, Nn, 1.0, A, M, x, 0.0, None, None) == N.INVALID_ARGUMENT
    assert L.cuopx_gemv_noalloc(99, 1, M, Nn, 1.0, A, M, x, 0.0, y, None) == N.UNSUPPORTED_TYPE
    # vector ops
    assert L.cuopx_axpy(-1, 1.0, 16, 1, 32, 1, None) == N.INVALID_ARGUMENT
    assert L.cuopx_axpy(4, 1.0, 16, 0, 32, 1, None) == N.INVALID_ARGUMENT
    assert L.cuopx_gather_column_blocks(N.F16, 2, 4, 4, 16, 64, 7, None) == N.INVALID_ARGUMENT
    # fused epilogue: unknown flags, bias flag without a bias vector
    assert L.cuopx_gemm_ex(N.F32, 0, 0, 4, 4, 4, 1.0, 16, 4, 16, 4, 0.0, 64, 4, None, 4, None) == N.INVALID_ARGUMENT
    assert L.cuopx_gemm_ex(N.F32, 0, 0, 4, 4, 4, 1.0, 16, 4, 16, 4, 0.0, 64, 4, None, N.EPI_BIAS,
                           None) == N.INVALID_ARGUMENT
    # fused all-gather: rank outside the world, too many ranks
    ptrs = (C.c_void_p * 2)(4096, 8192)
    assert L.cuopx_gemm_allgather(N.F16, 0, 0, 512, 256, 512, 1.0, 16, 512, 32, 256, ptrs, 2, 2, 512,
                                  None) == N.INVALID_ARGUMENT
    assert L.cuopx_gemm_allgather(N.F16, 0, 0, 512, 256, 512, 1.0, 16, 512, 32, 256, ptrs, 9, 0, 4608,
                                  None) == N.INVALID_ARGUMENT
    assert L.cuopx_peer_barrier(ptrs, 2, 5, None) == N.INVALID_ARGUMENT


def test_workspace_sizing_is_host_only():
    L = cx.lib()
    assert L.cuopx_gemv_workspace_size(N.F32, 0, 0, 100) == 0
    # transposed 8192^2 needs split-K partials; sizes are 256-byte multiples
    ws = L.cuopx_gemv_workspace_size(N.F32, 1, 8192, 8192)
    assert ws > 0 and ws % 256 == 0
    assert L.cuopx_vector_workspace_size(1 << 20) >= 1024 * 16


def test_last_kernel_defaults():
    assert isinstance(cx.last_kernel(), str)
    assert cx.launch_count() >= 0


def test_ops_refuse_cpu_tensors():
    import torch

    with pytest.raises(cx.CuopError):
        cx.gemm(torch.zeros(4, 4), torch.zeros(4, 4))
    with pytest.raises(cx.CuopError):
        cx.gemv(torch.zeros(4, 4), torch.zeros(4))


def test_tuning_table_parsing_without_gpu():
    L = cx.lib()
    names = []
    i = 0
    while L.cuopx_gemm_variant_name(i) is not None:
        names.append(L.cuopx_gemm_variant_name(i).decode())
        i += 1
    assert names[0] == "auto" and {"tc2", "tc_128x256", "tc_128x128", "tf32x3_128x64", "ffma", "generic"} <= set(names)
    try:
        assert L.cuopx_tuning_load(b"# comment only\n\n") == N.SUCCESS and L.cuopx_tuning_rows() == 0
        ok = b"bf16 0 0 256: 256: 256: 1:1 tc2   # trailing comment\nf32 * * * :255 * * ffma\n"
        assert L.cuopx_tuning_load(ok) == N.SUCCESS and L.cuopx_tuning_rows() == 2
        for bad in (b"bf16 0 0 256: 256: tc2\n", b"bf16 0 0 256: 256: 1: * bogus\n", b"x16 0 0 * * * * tc2\n",
                    b"f32 2 0 * * * * tc2\n", b"f32 0 0 9:1 * * * tc2\n", b"f32 0 0 1-9 * * * tc2\n"):
            assert L.cuopx_tuning_load(bad) == N.INVALID_ARGUMENT, bad
        assert L.cuopx_tuning_rows() == 2  # a rejected table leaves the loaded one in place
        assert L.cuopx_tuning_load_file(b"/nonexistent/table.txt") == N.INVALID_ARGUMENT
        assert L.cuopx_set_gemm_variant(b"not-a-variant") == N.INVALID_ARGUMENT
        assert L.cuopx_set_gemm_variant(b"ffma") == N.SUCCESS
    finally:
        L.cuopx_set_gemm_variant(None)
        L.cuopx_tuning_clear()
    assert L.cuopx_tuning_rows() == 0


def test_call_log_is_opt_in():
    """CUOPX_LOG=1 prints one line per C-ABI call; unset, nothing is printed."""
    import subprocess
    import sys

    code = ("import sys; sys.path.insert(0, %r); from cuop_b200 import _native as N; L = N.lib(); "
            "print(L.cuopx_gemm(0, 0, 0, -1, 4, 4, 1.0, 16, 4, 16, 4, 0.0, 16, 4, None), "
            "L.cuopx_gemv(0, 0, 4, 8, 1.0, 4096, 4, 8192, 0.0, 16384, None, 0, None), "
            "L.cuopx_gemm_ex(0, 0, 0, 4, 4, 4, 1.0, 16, 4, 16, 4, 0.0, 64, 4, None, 1, None))" % str(ROOT))
    on = subprocess.run([sys.executable, "-c", code], env={**__import__("os").environ, "CUOPX_LOG": "1"},
                        capture_output=True, text=True, timeout=120)
    assert on.returncode == 0 and on.stdout.split() == [str(N.INVALID_ARGUMENT)] * 3
    lines = [ln for ln in on.stderr.splitlines() if ln.startswith("cuopx: ")]
    assert len(lines) == 3 and all(ln.endswith("status 4001") for ln in lines), on.stderr
    assert lines[0].startswith("cuopx: cuopx_gemm -1 x 4 x 4")
    assert lines[1].startswith("cuopx: cuopx_gemv 4 x 8") and lines[2].startswith("cuopx: cuopx_gemm_ex 4 x 4 x 4")
    env = {k: v for k, v in __import__("os").environ.items() if k != "CUOPX_LOG"}
    off = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=120)
    assert off.returncode == 0 and "cuopx:" not in off.stderr



def test_last_cuda_error_starts_empty():
    """cuopx_last_cuda_error names the CUDA error behind a CUOPX_CUDA_ERROR;
    before any such failure on this thread it is "none" (no GPU needed)."""
    import threading

    seen = []
    t = threading.Thread(target=lambda: seen.append(cx.lib().cuopx_last_cuda_error().decode()))
    t.start()
    t.join()
    assert seen == ["none"]
