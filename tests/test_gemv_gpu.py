"""GEMV parity: CUDA kernels (through the C ABI) vs the CPU oracle and, at the
benchmark size, vs the reference's own Gemv<float> compiled from its sources.

Tolerance (fp32): ||y - r||_F / ||r||_F <= 1e-5 * sqrt(N)."""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

import cuop_b200 as cx
import oracle as O
from helpers import to_dev_f32

pytestmark = pytest.mark.gpu
GOLD = json.loads((Path(__file__).parent / "golden" / "known_answers.json").read_text())


def test_known_answer(dev):
    g = GOLD["gemv_2x3"]  # test/cuBlas/test_gemv/test_gemv.cpp:19-44
    A = to_dev_f32(np.array(g["A"]).reshape(2, 3), dev)
    y = cx.gemv(A, to_dev_f32(np.array(g["x"]), dev))
    np.testing.assert_allclose(y.cpu().numpy(), g["expected"], atol=g["tol"])


SHAPES = [(1, 1), (2, 3), (17, 33), (64, 8192), (8, 100_000), (4096, 64), (1000, 1000), (333, 4099), (2048, 2048)]


@pytest.mark.parametrize("trans", [False, True])
@pytest.mark.parametrize("M,N", SHAPES)
def test_f32_vs_oracle(dev, M, N, trans):
    A = O.uniform((N, M) if trans else (M, N), seed=M * 7 + N)
    x = O.uniform(N, seed=1)
    y0 = O.uniform(M, seed=2)
    ref = O.gemv_f32(A, x, y0, trans=trans, alpha=1.25, beta=-0.5)
    y = cx.gemv(to_dev_f32(A, dev), to_dev_f32(x, dev), to_dev_f32(y0, dev), trans=trans, alpha=1.25, beta=-0.5)
    err = O.rel_frobenius(y.cpu().numpy(), ref)
    assert err <= 1e-5 * np.sqrt(N), (err, cx.last_kernel())


@pytest.mark.parametrize("trans", [False, True])
def test_beta_zero_ignores_garbage_y(dev, trans):
    M, N = 300, 500
    A = O.uniform((N, M) if trans else (M, N), seed=3)
    x = O.uniform(N, seed=4)
    y = torch.full((M,), float("nan"), device=dev)
    cx.gemv(to_dev_f32(A, dev), to_dev_f32(x, dev), y, trans=trans, beta=0.0)
    assert torch.isfinite(y).all()
    assert O.rel_frobenius(y.cpu().numpy(), O.gemv_f32(A, x, trans=trans)) <= 1e-5 * np.sqrt(N)


@pytest.mark.parametrize("trans", [False, True])
def test_deterministic(dev, trans):
    M, N = 4096, 4096
    A = to_dev_f32(O.uniform((M, N), seed=5), dev)
    x = to_dev_f32(O.uniform(N, seed=6), dev)
    y1 = cx.gemv(A, x, trans=trans).clone()
    y2 = cx.gemv(A, x, trans=trans)
    assert torch.equal(y1, y2)


@pytest.mark.parametrize("dtype", [torch.float64, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("trans", [False, True])
def test_other_dtypes(dev, dtype, trans):
    M, N = 777, 1536
    A32 = O.uniform((N, M) if trans else (M, N), seed=9)
    x32 = O.uniform(N, seed=10)
    A = torch.from_numpy(A32).to(dev, dtype)
    x = torch.from_numpy(x32).to(dev, dtype)
    y = cx.gemv(A, x, trans=trans)
    ref = O.gemv_f64acc(A.float().cpu().numpy(), x.float().cpu().numpy(), trans=trans)
    tol = 1e-12 * np.sqrt(N) if dtype == torch.float64 else 1e-2
    err = O.rel_frobenius(y.double().cpu().numpy(), ref) if dtype == torch.float64 else \
        O.max_relative(y.float().cpu().numpy(), ref)
    assert err <= tol, err


def test_without_workspace_falls_back(dev):
    """With no scratch the single-pass kernels run; results still meet tolerance."""
    from cuop_b200 import _native as N

    M, N_ = 8192, 8192
    A32 = O.uniform((N_, M), seed=11)
    x32 = O.uniform(N_, seed=12)
    A, x = to_dev_f32(A32, dev), to_dev_f32(x32, dev)
    y = torch.empty(M, device=dev)
    rc = N.lib().cuopx_gemv(N.F32, 1, M, N_, 1.0, A.data_ptr(), M, x.data_ptr(), 0.0, y.data_ptr(), None, 0,
                            torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    assert cx.last_kernel() == "gemv_t_single"
    ref = O.gemv_f32(A32, x32, trans=True)
    assert O.rel_frobenius(y.cpu().numpy(), ref) <= 1e-5 * np.sqrt(N_)


@pytest.mark.parametrize("trans", [False, True])
def test_benchmark_size_vs_cpu_and_reference_operator(dev, trans):
    """C2: 8192 x 8192 fp32, A, x ~ U[-1,1) seeds 0/1 — ours vs the CPU
    restatement vs the reference's Gemv<float>::Forward on the same GPU."""
    M = N_ = 8192
    A32 = O.uniform((M, N_), seed=0)
    x32 = O.uniform(N_, seed=1)
    A, x = to_dev_f32(A32, dev), to_dev_f32(x32, dev)
    y = cx.gemv(A, x, trans=trans)
    assert cx.last_kernel() == ("gemv_t_lsu" if trans else "gemv_n_xreg")
    cpu = O.gemv_f32(A32, x32, trans=trans)
    exact = O.gemv_f64acc(A32, x32, trans=trans)
    tol = 1e-5 * np.sqrt(N_)
    assert O.rel_frobenius(y.cpu().numpy(), exact) <= tol
    assert O.rel_frobenius(cpu, exact) <= tol
    if O.ref_available():
        yr = torch.zeros(M, device=dev)
        torch.cuda.synchronize()
        rc = O.ref_lib().ref_gemv_f32(int(trans), M, N_, 1.0, A.data_ptr(), x.data_ptr(), 0.0, yr.data_ptr())
        assert rc == 0
        assert O.rel_frobenius(yr.cpu().numpy(), exact) <= tol
        assert O.rel_frobenius(y.cpu().numpy(), yr.cpu().numpy()) <= tol


@pytest.mark.parametrize("M,N", [(1000, 8192), (256, 100000), (8192, 17), (8192, 4099), (4352, 777)])
def test_transposed_strip_and_split_edges(dev, M, N):
    """Partial last strip (M not a multiple of the strip width), many splits
    with a ragged last one, a single split, and rows not a multiple of the
    per-split batch."""
    A = O.uniform((N, M), seed=21)
    x = O.uniform(N, seed=22)
    y = cx.gemv(to_dev_f32(A, dev), to_dev_f32(x, dev), trans=True)
    exact = O.gemv_f64acc(A, x, trans=True)
    assert O.rel_frobenius(y.cpu().numpy(), exact) <= 1e-5 * np.sqrt(N)
    assert cx.device_error() == 0


@pytest.mark.parametrize("trans", [False, True])
def test_result_into_pinned_host_memory(dev, trans):
    """y in pinned host memory: the kernel writes the result there directly,
    bit-identical to a device y."""
    M, N = 2048, 3072
    A = to_dev_f32(O.uniform((N, M) if trans else (M, N), seed=23), dev)
    x = to_dev_f32(O.uniform(N, seed=24), dev)
    y_dev = cx.gemv(A, x, trans=trans)
    y_host = torch.full((M,), float("nan")).pin_memory()
    cx.gemv(A, x, y_host, trans=trans)
    torch.cuda.synchronize()
    assert torch.equal(y_host, y_dev.cpu())


def test_outputs_that_the_device_cannot_reach_are_refused(dev):
    A = torch.zeros(64, 64, device=dev)
    x = torch.zeros(64, device=dev)
    with pytest.raises(cx.CuopError):
        cx.gemv(A, x, torch.zeros(64))  # pageable host memory
    with pytest.raises(cx.CuopError):
        cx.gemv(A, x.double())  # x of another dtype
    with pytest.raises(cx.CuopError):
        cx.gemm(A.half(), A.half(), torch.zeros(64, 64, dtype=torch.half))
    with pytest.raises(cx.CuopError):
        cx.batched_gemm(A.half()[None], A.half()[None], torch.zeros(1, 64, 64, dtype=torch.half))
