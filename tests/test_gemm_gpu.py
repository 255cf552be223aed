"""GEMM parity through the C ABI.

fp32 / fp64 on the FFMA kernels: every output is the same ascending-k fma
chain as the CPU oracle, so results must be BIT-IDENTICAL to it; the bound
||C-R||_F/||R||_F <= 1e-5*sqrt(K) is checked against an fp64 product too.
fp32 on the tensor cores (3xTF32, the default for >= 256^3): the same bound
against the fp64 product.
fp16 / bf16 (tcgen05 kernels): max|C-R| / max|R| <= 1e-2 against the oracle
(fp32 products and sums, one rounding)."""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

import cuop_b200 as cx
import oracle as O
from helpers import TDT, forced_variant, fp32_reference_gpu, lowp_bits, to_dev_f32, to_dev_lowp

pytestmark = pytest.mark.gpu
GOLD = json.loads((Path(__file__).parent / "golden" / "known_answers.json").read_text())
LOWP_TOL = 1e-2


def test_known_answer_all_dtypes(dev):
    g = GOLD["gemm_2x3x4"]  # test/cuBlas/test_gemm/test_gemm.cpp:19-43
    A = np.array(g["A"], np.float32).reshape(2, 3)
    B = np.array(g["B"], np.float32).reshape(3, 4)
    for dtype in (torch.float32, torch.float64, torch.float16, torch.bfloat16):
        C = cx.gemm(torch.from_numpy(A).to(dev, dtype), torch.from_numpy(B).to(dev, dtype))
        np.testing.assert_allclose(C.double().cpu().numpy().ravel(), g["expected"], atol=g["tol"])


F32_CASES = [
    (1, 1, 1, False, False), (2, 3, 4, False, False), (33, 17, 65, False, False), (33, 17, 65, True, False),
    (33, 17, 65, False, True), (33, 17, 65, True, True), (128, 128, 128, False, False), (200, 300, 64, False, False),
    (257, 129, 1000, False, False), (64, 64, 3, False, False), (512, 96, 77, True, True),
]


@pytest.mark.parametrize("M,N,K,tA,tB", F32_CASES)
def test_f32_bit_exact_vs_oracle(dev, fp32_ffma, M, N, K, tA, tB):
    A = O.uniform((K, M) if tA else (M, K), seed=M + 1)
    B = O.uniform((N, K) if tB else (K, N), seed=N + 2)
    C0 = O.uniform((M, N), seed=3)
    # alpha, beta not powers of two: any other epilogue rounding shows in the last bit
    al, be = float(np.float32(0.7)), float(np.float32(1.3))
    ref = O.gemm_f32(A, B, C0, transA=tA, transB=tB, alpha=al, beta=be)
    C = cx.gemm(to_dev_f32(A, dev), to_dev_f32(B, dev), to_dev_f32(C0, dev), transA=tA, transB=tB, alpha=al, beta=be)
    got = C.cpu().numpy()
    np.testing.assert_array_equal(got, ref, err_msg=cx.last_kernel())
    exact = al * ((A.T if tA else A).astype(np.float64) @ (B.T if tB else B).astype(np.float64)) + be * C0
    assert O.rel_frobenius(got, exact) <= 1e-5 * np.sqrt(K)


def test_f32_fast_kernel_selected(dev, fp32_ffma):
    A = to_dev_f32(O.uniform((512, 512), seed=1), dev)
    B = to_dev_f32(O.uniform((512, 512), seed=2), dev)
    cx.gemm(A, B)
    assert cx.last_kernel().startswith("gemm_f32_")


def test_f64_bit_exact_vs_oracle(dev):
    A = np.asarray(O.uniform((70, 90), seed=4), np.float64)
    B = np.asarray(O.uniform((90, 50), seed=5), np.float64)
    C = cx.gemm(torch.from_numpy(A).to(dev), torch.from_numpy(B).to(dev))
    np.testing.assert_array_equal(C.cpu().numpy(), O.gemm_f64(A, B))


def test_c1_fp32_1024_ffma_bit_exact(dev, fp32_ffma):
    """C1 on the FFMA kernel: bit-identical to the oracle's ascending-k chain."""
    n = 1024
    A32 = O.uniform((n, n), seed=0)
    B32 = O.uniform((n, n), seed=1)
    C = cx.gemm(to_dev_f32(A32, dev), to_dev_f32(B32, dev))
    assert cx.last_kernel().startswith("gemm_f32_")
    np.testing.assert_array_equal(C.cpu().numpy(), O.gemm_f32(A32, B32))


def test_c1_fp32_1024_vs_oracle_and_reference_operator(dev):
    """C1: fp32 1024^3, A,B ~ U[-1,1) seeds 0/1, C zero, alpha=1 beta=0 —
    default path (3xTF32), the CPU oracle and the reference's own Gemm<float>
    all within 1e-5*sqrt(K) of the fp64 product."""
    n = 1024
    A32 = O.uniform((n, n), seed=0)
    B32 = O.uniform((n, n), seed=1)
    A, B = to_dev_f32(A32, dev), to_dev_f32(B32, dev)
    C = cx.gemm(A, B)
    assert cx.last_kernel().startswith("gemm_tf32x3_"), cx.last_kernel()
    cpu = O.gemm_f32(A32, B32)
    exact = A32.astype(np.float64) @ B32.astype(np.float64)
    tol = 1e-5 * np.sqrt(n)
    assert O.rel_frobenius(cpu, exact) <= tol
    err = O.rel_frobenius(C.cpu().numpy(), exact)
    assert err <= tol
    assert err <= 0.1 * tol  # 3xTF32 sits at least 10x inside the bound
    if O.ref_available():
        Cr = torch.zeros(n, n, device=dev)
        torch.cuda.synchronize()
        assert O.ref_lib().ref_gemm_f32(0, 0, n, n, n, 1.0, A.data_ptr(), B.data_ptr(), 0.0, Cr.data_ptr()) == 0
        ref_gpu = Cr.cpu().numpy()
        assert O.rel_frobenius(ref_gpu, exact) <= tol
        # The reference's blocked kernel is the oracle's ascending-k fma chain.
        assert O.rel_frobenius(ref_gpu, cpu) <= 1e-6
        assert O.rel_frobenius(C.cpu().numpy(), ref_gpu) <= tol


X3_CASES = [
    (256, 256, 256, False, False), (1024, 512, 768, False, False), (300, 200, 500, False, False),
    (512, 384, 256, True, False), (512, 384, 256, False, True), (512, 384, 256, True, True),
    (2048, 2048, 2048, False, False), (4096, 96, 4100, False, False),
]


@pytest.mark.parametrize("M,N,K,tA,tB", X3_CASES)
def test_f32_tf32x3_within_tolerance(dev, M, N, K, tA, tB):
    A = O.uniform((K, M) if tA else (M, K), seed=M + 5)
    B = O.uniform((N, K) if tB else (K, N), seed=N + 6)
    C0 = O.uniform((M, N), seed=7)
    C = cx.gemm(to_dev_f32(A, dev), to_dev_f32(B, dev), to_dev_f32(C0, dev), transA=tA, transB=tB, alpha=0.75,
                beta=-0.5)
    assert cx.last_kernel().startswith("gemm_tf32x3_"), cx.last_kernel()
    exact = 0.75 * ((A.T if tA else A).astype(np.float64) @ (B.T if tB else B).astype(np.float64)) - 0.5 * C0
    err = O.rel_frobenius(C.cpu().numpy(), exact)
    assert err <= 1e-5 * np.sqrt(K), err
    assert err <= 0.1 * 1e-5 * np.sqrt(K), err  # at least 10x inside the required bound


def test_f32_tf32x3_batched_and_deterministic(dev):
    A = to_dev_f32(O.uniform((6, 256, 192), seed=1), dev)
    B = to_dev_f32(O.uniform((6, 192, 320), seed=2), dev)
    C1 = cx.batched_gemm(A, B)
    assert cx.last_kernel().startswith("gemm_tf32x3_")
    C2 = cx.batched_gemm(A, B)
    assert torch.equal(C1, C2)
    exact = np.einsum("bmk,bkn->bmn", A.double().cpu().numpy(), B.double().cpu().numpy())
    assert O.rel_frobenius(C1.cpu().numpy(), exact) <= 0.1 * 1e-5 * np.sqrt(192)


def test_fp32_mode_switch_validates():
    from cuop_b200 import _native as N

    assert N.lib().cuopx_set_fp32_gemm_mode(7) == N.INVALID_ARGUMENT
    assert N.lib().cuopx_get_fp32_gemm_mode() == N.FP32_AUTO


LOWP_CASES = [
    (128, 256, 64, False, False), (256, 512, 128, False, False), (300, 504, 200, False, False),
    (129, 264, 72, False, False), (1000, 1000, 1000, False, False), (512, 384, 4096, False, False),
    (256, 384, 192, True, False), (256, 384, 192, False, True), (256, 384, 192, True, True),
    (384, 136, 320, True, True), (64, 128, 64, False, False), (2048, 2048, 512, False, False),
]


@pytest.mark.parametrize("dt", [O.F16, O.BF16])
@pytest.mark.parametrize("M,N,K,tA,tB", LOWP_CASES)
def test_lowp_tcgen05_vs_oracle(dev, dt, M, N, K, tA, tB):
    A = O.to_lowp(O.normal((K, M) if tA else (M, K), seed=M) / np.sqrt(K), dt)
    B = O.to_lowp(O.normal((N, K) if tB else (K, N), seed=N + 7), dt)
    ref = O.gemm_lowp(dt, A, B, transA=tA, transB=tB)
    C = cx.gemm(to_dev_lowp(A, dt, dev), to_dev_lowp(B, dt, dev), transA=tA, transB=tB)
    assert cx.last_kernel().startswith("gemm_tc_"), cx.last_kernel()
    err = O.max_relative(O.from_lowp(lowp_bits(C), dt), O.from_lowp(ref, dt))
    assert err <= LOWP_TOL, (err, cx.last_kernel())


PAIR_CASES = [  # the two-SM (cta_group::2) kernel, forced (ragged and transposed shapes)
    (4096, 2560, 512, False, False), (4000, 2600, 520, False, False), (2560, 4096, 256, True, False),
    (2560, 4096, 256, False, True), (2560, 4096, 256, True, True), (3072, 3072, 1000, False, False),
]


@pytest.mark.parametrize("variant,kernel", [("tc2", "gemm_tc2_256x256"), ("tc2_256x512", "gemm_tc2_256x512"),
                                            ("tc2_256x128", "gemm_tc2_256x128")])
@pytest.mark.parametrize("dt", [O.F16, O.BF16])
@pytest.mark.parametrize("M,N,K,tA,tB", PAIR_CASES)
def test_lowp_pair_kernel_vs_oracle(dev, dt, M, N, K, tA, tB, variant, kernel):
    A = O.to_lowp(O.normal((K, M) if tA else (M, K), seed=M + 11) / np.sqrt(K), dt)
    B = O.to_lowp(O.normal((N, K) if tB else (K, N), seed=N + 13), dt)
    C0 = O.to_lowp(O.normal((M, N), seed=17), dt)
    Cd = to_dev_lowp(C0, dt, dev)
    with forced_variant(variant):
        cx.gemm(to_dev_lowp(A, dt, dev), to_dev_lowp(B, dt, dev), Cd, transA=tA, transB=tB, alpha=1.5, beta=0.5)
    assert cx.last_kernel() == kernel, cx.last_kernel()
    full = 1.5 * fp32_reference_gpu(to_dev_lowp(A, dt, dev), to_dev_lowp(B, dt, dev), tA, tB) + \
        0.5 * to_dev_lowp(C0, dt, dev).float()
    assert O.max_relative(Cd.float().cpu().numpy(), full.cpu().numpy()) <= LOWP_TOL
    rows = np.array([0, 1, 255, 256, M - 1])
    ref = O.gemm_lowp(dt, A[:, rows] if tA else A[rows], B, C0[rows], transA=tA, transB=tB, alpha=1.5, beta=0.5)
    got = O.from_lowp(lowp_bits(Cd[torch.as_tensor(rows, device=dev)]), dt)
    assert O.max_relative(got, O.from_lowp(ref, dt)) <= LOWP_TOL


@pytest.mark.parametrize("M,N,K,kernel", [(8192, 8192, 4096, "gemm_tc2_256x512"), (8192, 1024, 8192, "gemm_tc2_256x512"),
                                           (4096, 1024, 8192, "gemm_tc2_256x256"), (4096, 28672, 8192, "gemm_tc2_256x512"),
                                           (1024, 8192, 4096, "gemm_tc2_256x512"), (8192, 8192, 1024, "gemm_tc_128x256")])
def test_pair_tile_width_follows_size(dev, M, N, K, kernel):
    """Built-in choice by waves of pair tiles: 256 x 512 tiles unless they
    leave the SM pairs idler than 256 x 256 tiles would; short K loops on the
    1-SM kernel.  Every choice agrees with an fp32 reference on sampled rows
    and columns."""
    g = torch.Generator(device=dev).manual_seed(M + N + K)
    A = (torch.randn(M, K, device=dev, generator=g) / np.sqrt(K)).bfloat16()
    B = torch.randn(K, N, device=dev, generator=g).bfloat16()
    C = cx.gemm(A, B)
    assert cx.last_kernel() == kernel, cx.last_kernel()
    rows = torch.tensor(sorted({r for r in (0, 1, 255, 256, 511, 4095, M - 1) if r < M}), device=dev)
    ref = A[rows].float() @ B.float()
    assert O.max_relative(C[rows].float().cpu().numpy(), ref.cpu().numpy()) <= LOWP_TOL
    cols = torch.tensor(sorted({c for c in (0, 255, 256, 511, 512, N - 1) if c < N}), device=dev)
    ref_c = A.float() @ B[:, cols].float()
    assert O.max_relative(C[:, cols].float().cpu().numpy(), ref_c.cpu().numpy()) <= LOWP_TOL


@pytest.mark.parametrize("dt", [O.F16, O.BF16])
def test_lowp_alpha_beta(dev, dt):
    M, N, K = 320, 640, 256
    A = O.to_lowp(O.normal((M, K), seed=1) / np.sqrt(K), dt)
    B = O.to_lowp(O.normal((K, N), seed=2), dt)
    C0 = O.to_lowp(O.normal((M, N), seed=3), dt)
    ref = O.gemm_lowp(dt, A, B, C0, alpha=0.75, beta=-1.25)
    Cd = to_dev_lowp(C0, dt, dev)
    cx.gemm(to_dev_lowp(A, dt, dev), to_dev_lowp(B, dt, dev), Cd, alpha=0.75, beta=-1.25)
    assert cx.last_kernel().startswith("gemm_tc_")
    assert O.max_relative(O.from_lowp(lowp_bits(Cd), dt), O.from_lowp(ref, dt)) <= LOWP_TOL


def test_lowp_strided_leading_dims(dev):
    """Row-major views with padded leading dimensions (multiples of 8)."""
    dt = O.BF16
    M, N, K = 200, 192, 136
    Ab = O.to_lowp(O.normal((M, K + 24), seed=4), dt)
    Bb = O.to_lowp(O.normal((K, N + 8), seed=5), dt)
    A = to_dev_lowp(Ab, dt, dev)[:, :K]
    B = to_dev_lowp(Bb, dt, dev)[:, :N]
    Cbig = torch.zeros(M, N + 16, device=dev, dtype=torch.bfloat16)
    C = Cbig[:, :N]
    cx.gemm(A, B, C)
    assert cx.last_kernel().startswith("gemm_tc_")
    ref = O.gemm_lowp(dt, np.ascontiguousarray(Ab[:, :K]), np.ascontiguousarray(Bb[:, :N]))
    assert O.max_relative(O.from_lowp(lowp_bits(C.contiguous()), dt), O.from_lowp(ref, dt)) <= LOWP_TOL
    assert torch.count_nonzero(Cbig[:, N:]) == 0  # padding columns untouched


def test_lowp_unaligned_uses_generic(dev):
    dt = O.F16
    A = O.to_lowp(O.normal((50, 37), seed=1), dt)
    B = O.to_lowp(O.normal((37, 45), seed=2), dt)
    C = cx.gemm(to_dev_lowp(A, dt, dev), to_dev_lowp(B, dt, dev))
    assert cx.last_kernel() == "gemm_simt_generic"
    ref = O.gemm_lowp(dt, A, B)
    assert O.max_relative(O.from_lowp(lowp_bits(C), dt), O.from_lowp(ref, dt)) <= LOWP_TOL


def _rows_cols_check(C, A32, B32, rows, cols):
    """Max-relative error of complete rows and complete columns of C against
    the fp64 oracle (the worse of the two sets)."""
    R, Q = O.gemm_rows_cols_f64(A32, B32, rows, cols)
    got_rows = C[torch.as_tensor(rows, device=C.device)].float().cpu().numpy()
    got_cols = C[:, torch.as_tensor(cols, device=C.device)].float().cpu().numpy()
    return max(O.max_relative(got_rows, R), O.max_relative(got_cols, Q))


def test_c3_fp16_8192_full(dev):
    """C3: fp16 8192^3, A,B ~ N(0,1)/sqrt(K), fp32 accumulate, fp16 out."""
    n = 8192
    dt = O.F16
    A16 = O.to_lowp(O.normal((n, n), seed=0) / np.sqrt(n), dt)
    B16 = O.to_lowp(O.normal((n, n), seed=1) / np.sqrt(n), dt)
    A, B = to_dev_lowp(A16, dt, dev), to_dev_lowp(B16, dt, dev)
    C = cx.gemm(A, B)
    assert cx.last_kernel() == "gemm_tc2_256x512"
    full = fp32_reference_gpu(A, B)
    assert O.max_relative(C.float().cpu().numpy(), full.cpu().numpy()) <= LOWP_TOL
    # 256 complete rows and 256 complete columns against the fp64 oracle
    rng = np.random.default_rng(0)
    rows = np.sort(rng.choice(n, 256, replace=False))
    cols = np.sort(rng.choice(n, 256, replace=False))
    assert _rows_cols_check(C, O.from_lowp(A16, dt), O.from_lowp(B16, dt), rows, cols) <= LOWP_TOL


def test_c5_bf16_linear_full(dev):
    """C5: X 4096x8192 ~ N(0,1), W 8192x28672 ~ N(0,0.02), bf16 out."""
    M, K, N = 4096, 8192, 28672
    dt = O.BF16
    X16 = O.to_lowp(O.normal((M, K), seed=0), dt)
    W16 = O.to_lowp(O.normal((K, N), seed=1, std=0.02), dt)
    X, W = to_dev_lowp(X16, dt, dev), to_dev_lowp(W16, dt, dev)
    Y = cx.gemm(X, W)
    full = fp32_reference_gpu(X, W)
    assert O.max_relative(Y.float().cpu().numpy(), full.cpu().numpy()) <= LOWP_TOL
    del full
    # 256 complete rows and 256 complete columns against the fp64 oracle
    rng = np.random.default_rng(1)
    rows = np.sort(rng.choice(M, 256, replace=False))
    cols = np.sort(rng.choice(N, 256, replace=False))
    assert _rows_cols_check(Y, O.from_lowp(X16, dt), O.from_lowp(W16, dt), rows, cols) <= LOWP_TOL


def test_deterministic_lowp(dev):
    dt = O.BF16
    A = to_dev_lowp(O.to_lowp(O.normal((1024, 2048), seed=1), dt), dt, dev)
    B = to_dev_lowp(O.to_lowp(O.normal((2048, 1536), seed=2), dt), dt, dev)
    assert torch.equal(cx.gemm(A, B), cx.gemm(A, B))


TWO_PER_SM_CASES = [  # (batch, M, N, K, transA, transB)
    (1, 300, 504, 200, False, False), (3, 256, 384, 192, True, False), (3, 256, 384, 192, False, True),
    (2, 384, 136, 320, True, True), (512, 128, 128, 64, False, False), (37, 200, 136, 72, False, False),
]


@pytest.mark.parametrize("dt", [O.F16, O.BF16])
@pytest.mark.parametrize("batch,M,N,K,tA,tB", TWO_PER_SM_CASES)
def test_lowp_two_ctas_per_sm_variant(dev, dt, batch, M, N, K, tA, tB):
    """The 1-SM kernel with two CTAs per SM (128 x 128 tiles, two stages, or
    128 x 64 tiles, three stages; 256 TMEM columns per CTA) runs, for every
    output, the same MMAs over K in the same order as the one-CTA kernel:
    bit-identical results, and within tolerance of the oracle."""
    A = O.to_lowp(O.normal((batch, K, M) if tA else (batch, M, K), seed=M + batch) / np.sqrt(K), dt)
    B = O.to_lowp(O.normal((batch, N, K) if tB else (batch, K, N), seed=N + 3), dt)
    C0 = O.to_lowp(O.normal((batch, M, N), seed=K), dt)
    outs = []
    for variant, kernel in (("tc_128x128_2cta", "gemm_tc_128x128_2cta"), ("tc_128x128", "gemm_tc_128x128"),
                            ("tc_128x64_2cta", "gemm_tc_128x64_2cta")):
        Cd = to_dev_lowp(C0, dt, dev)
        with forced_variant(variant):
            cx.batched_gemm(to_dev_lowp(A, dt, dev), to_dev_lowp(B, dt, dev), Cd, transA=tA, transB=tB,
                            alpha=0.75, beta=-0.5)
        assert cx.last_kernel() == kernel, cx.last_kernel()
        outs.append(Cd)
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])
    for b in sorted({0, batch - 1}):
        ref = O.gemm_lowp(dt, A[b], B[b], C0[b], transA=tA, transB=tB, alpha=0.75, beta=-0.5)
        assert O.max_relative(O.from_lowp(lowp_bits(outs[0][b]), dt), O.from_lowp(ref, dt)) <= LOWP_TOL


SPLITK_CASES = [  # (batch, M, N, K, transA, transB)
    (1, 1024, 1024, 1024, False, False), (1, 512, 512, 512, False, False), (1, 384, 320, 1000, False, False),
    (1, 256, 192, 416, True, False), (1, 256, 264, 96, False, True), (3, 256, 128, 384, True, True),
]


@pytest.mark.parametrize("batch,M,N,K,tA,tB", SPLITK_CASES)
def test_f32_tf32x3_split_k_pair(dev, batch, M, N, K, tA, tB):
    """3xTF32 with K split over a CTA pair (partial sums exchanged through
    distributed shared memory, added in a fixed order): within a tenth of the
    fp32 bound of an fp64 product, with alpha/beta and a fused bias + ReLU,
    and the same bits on every run."""
    A32 = O.uniform((batch, K, M) if tA else (batch, M, K), seed=M + K)
    B32 = O.uniform((batch, N, K) if tB else (batch, K, N), seed=N + 1)
    C32 = O.uniform((batch, M, N), seed=7)
    A, B = to_dev_f32(A32, dev), to_dev_f32(B32, dev)
    outs = []
    for _ in range(2):
        Cd = to_dev_f32(C32, dev)
        with forced_variant("tf32x3_128x128_k2"):
            cx.batched_gemm(A, B, Cd, transA=tA, transB=tB, alpha=0.75, beta=-0.5)
        assert cx.last_kernel() == "gemm_tf32x3_128x128_k2", cx.last_kernel()
        outs.append(Cd)
    assert torch.equal(outs[0], outs[1])
    opA = np.swapaxes(A32, 1, 2) if tA else A32
    opB = np.swapaxes(B32, 1, 2) if tB else B32
    exact = 0.75 * np.einsum("bmk,bkn->bmn", opA.astype(np.float64), opB.astype(np.float64)) - 0.5 * C32
    assert O.rel_frobenius(outs[0].cpu().numpy(), exact) <= 0.1 * 1e-5 * np.sqrt(K)
    if batch == 1 and not tA and not tB:
        bias = to_dev_f32(O.uniform(N, seed=9), dev)
        with forced_variant("tf32x3_128x128_k2"):
            Cr = cx.gemm(A[0], B[0], bias=bias, relu=True)
        ref = np.maximum(A32[0].astype(np.float64) @ B32[0].astype(np.float64) + bias.double().cpu().numpy(), 0.0)
        assert O.rel_frobenius(Cr.cpu().numpy(), ref) <= 0.1 * 1e-5 * np.sqrt(K)


PAIR_CASES = [  # (batch, M, N, K, transB); A is K-major (the pair kernel splits A into TMEM)
    (1, 1024, 1024, 1024, False), (1, 512, 512, 512, False), (1, 300, 200, 500, False),
    (1, 384, 320, 1000, True), (2, 256, 264, 96, True), (3, 200, 136, 384, False), (1, 128, 128, 96, False),
]


@pytest.mark.parametrize("batch,M,N,K,tB", PAIR_CASES)
def test_f32_tf32x3_pair_split_k(dev, batch, M, N, K, tB):
    """3xTF32 on CTA pairs (tcgen05 cta_group::2, 256 x 128 tiles, each CTA
    splitting its A rows into its own TMEM and holding half of B) with K
    split over two pairs: within a tenth of the fp32 bound of an fp64
    product, with alpha/beta, ragged M/N/K and a fused bias + ReLU, and the
    same bits on every run."""
    A32 = O.uniform((batch, M, K), seed=M + K)
    B32 = O.uniform((batch, N, K) if tB else (batch, K, N), seed=N + 1)
    C32 = O.uniform((batch, M, N), seed=7)
    A, B = to_dev_f32(A32, dev), to_dev_f32(B32, dev)
    outs = []
    for _ in range(2):
        Cd = to_dev_f32(C32, dev)
        with forced_variant("tf32x3_256x128_pair"):
            cx.batched_gemm(A, B, Cd, transB=tB, alpha=0.75, beta=-0.5)
        assert cx.last_kernel() == "gemm_tf32x3_256x128_pair_k2", cx.last_kernel()
        outs.append(Cd)
    assert cx.device_error() == 0
    assert torch.equal(outs[0], outs[1])
    opB = np.swapaxes(B32, 1, 2) if tB else B32
    exact = 0.75 * np.einsum("bmk,bkn->bmn", A32.astype(np.float64), opB.astype(np.float64)) - 0.5 * C32
    assert O.rel_frobenius(outs[0].cpu().numpy(), exact) <= 0.1 * 1e-5 * np.sqrt(K)
    if batch == 1 and not tB:
        bias = to_dev_f32(O.uniform(N, seed=9), dev)
        with forced_variant("tf32x3_256x128_pair"):
            Cr = cx.gemm(A[0], B[0], bias=bias, relu=True)
        assert cx.last_kernel() == "gemm_tf32x3_256x128_pair_k2", cx.last_kernel()
        ref = np.maximum(A32[0].astype(np.float64) @ B32[0].astype(np.float64) + bias.double().cpu().numpy(), 0.0)
        assert O.rel_frobenius(Cr.cpu().numpy(), ref) <= 0.1 * 1e-5 * np.sqrt(K)


def test_f32_tf32x3_pair_falls_back_for_mn_major_a(dev):
    """The pair kernel takes K-major A only: a transposed A forced onto it
    runs the one-CTA split instead, with the same accuracy."""
    A32 = O.uniform((512, 256), seed=3)  # A^T stored: (K, M)
    B32 = O.uniform((512, 384), seed=4)
    with forced_variant("tf32x3_256x128_pair"):
        C = cx.gemm(to_dev_f32(A32, dev), to_dev_f32(B32, dev), transA=True)
    assert cx.last_kernel() == "gemm_tf32x3_128x128_k2", cx.last_kernel()
    exact = A32.T.astype(np.float64) @ B32.astype(np.float64)
    assert O.rel_frobenius(C.cpu().numpy(), exact) <= 0.1 * 1e-5 * np.sqrt(512)


def test_f32_1024_default_takes_pair_split_k(dev):
    """C1 (1024^3: 32 tiles of 256 x 128) fills the part with CTA pairs and K
    split over two pairs (128 CTAs)."""
    A = to_dev_f32(O.uniform((1024, 1024), seed=0), dev)
    B = to_dev_f32(O.uniform((1024, 1024), seed=1), dev)
    cx.gemm(A, B)
    assert cx.last_kernel() == "gemm_tf32x3_256x128_pair_k2"
