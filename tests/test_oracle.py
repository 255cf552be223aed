"""CPU tests of the oracle: pinned to the reference's known answers, the
rounding helpers checked exhaustively, the generator's determinism, and the
restated GEMM/GEMV math against an independent numpy fp64 product."""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle as O

GOLD = json.loads((Path(__file__).parent / "golden" / "known_answers.json").read_text())


# --------------------------------------------------------------- known answers
def test_known_answer_gemm():
    g = GOLD["gemm_2x3x4"]  # test/cuBlas/test_gemm/test_gemm.cpp:19-43
    A = np.array(g["A"], np.float32).reshape(g["M"], g["K"])
    B = np.array(g["B"], np.float32).reshape(g["K"], g["N"])
    C = O.gemm_f32(A, B, alpha=g["alpha"], beta=g["beta"])
    np.testing.assert_allclose(C.ravel(), g["expected"], atol=g["tol"])


def test_known_answer_gemv():
    g = GOLD["gemv_2x3"]  # test/cuBlas/test_gemv/test_gemv.cpp:19-44
    A = np.array(g["A"], np.float32).reshape(g["M"], g["N"])
    y = O.gemv_f32(A, np.array(g["x"], np.float32))
    np.testing.assert_allclose(y, g["expected"], atol=g["tol"])


def test_known_answer_matmul_2d_and_batch():
    g = GOLD["matmul_2d"]  # test/cuDNN/test_matmul/test_matmul.cpp:21-39
    A = np.array(g["A"], np.float32).reshape(g["M"], g["K"])
    B = np.array(g["B"], np.float32).reshape(g["K"], g["N"])
    np.testing.assert_allclose(O.gemm_f32(A, B).ravel(), g["expected"], atol=g["tol"])
    g = GOLD["matmul_batch3d"]  # test_matmul.cpp:41-67
    A = np.array(g["A"], np.float32).reshape(g["batch"], g["M"], g["K"])
    B = np.array(g["B"], np.float32).reshape(g["batch"], g["K"], g["N"])
    np.testing.assert_allclose(O.gemm_batched_f32(A, B).ravel(), g["expected"], atol=g["tol"])


def test_known_answer_lowp():
    """The same cases in fp16/bf16 are exact (small integers)."""
    g = GOLD["gemm_2x3x4"]
    for dt in (O.F16, O.BF16):
        A = O.to_lowp(np.array(g["A"], np.float32).reshape(2, 3), dt)
        B = O.to_lowp(np.array(g["B"], np.float32).reshape(3, 4), dt)
        C = O.from_lowp(O.gemm_lowp(dt, A, B), dt)
        np.testing.assert_array_equal(C.ravel(), g["expected"])


# --------------------------------------------------------------- rounding
def test_lowp_roundtrip_exhaustive():
    """Every fp16 / bf16 bit pattern survives widen -> narrow (NaNs stay NaN)."""
    bits = np.arange(65536, dtype=np.uint16)
    for dt in (O.F16, O.BF16):
        f = O.from_lowp(bits, dt)
        back = O.to_lowp(f, dt)
        nan = np.isnan(f)
        np.testing.assert_array_equal(back[~nan], bits[~nan])
        assert np.all(np.isnan(O.from_lowp(back[nan], dt)))


def test_widening_matches_torch():
    bits = np.arange(65536, dtype=np.uint16)
    f16 = O.from_lowp(bits, O.F16)
    ref16 = torch.from_numpy(bits.view(np.int16)).view(torch.float16).float().numpy()
    np.testing.assert_array_equal(np.isnan(f16), np.isnan(ref16))
    ok = ~np.isnan(ref16)
    np.testing.assert_array_equal(f16[ok], ref16[ok])
    bf = O.from_lowp(bits, O.BF16)
    refb = torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).float().numpy()
    ok = ~np.isnan(refb)
    np.testing.assert_array_equal(bf[ok], refb[ok])


@pytest.mark.parametrize("dt,tdt", [(O.F16, torch.float16), (O.BF16, torch.bfloat16)])
def test_rne_matches_torch(dt, tdt):
    rng = np.random.default_rng(7)
    # random bit patterns cover normals, subnormals, overflow and ties
    x = rng.integers(0, 2**32, size=2_000_000, dtype=np.uint64).astype(np.uint32).view(np.float32)
    x = x[~np.isnan(x)]
    edge = np.array([0.0, -0.0, 65504.0, 65519.996, 65520.0, 65536.0, 2**-24, 2**-25, 2**-25 * 1.0000001,
                     3 * 2**-26, 2**-14, 2**-14 * (1 - 2**-11), 1.0 + 2**-11, 1.0 + 3 * 2**-11, np.inf, -np.inf],
                    np.float32)
    x = np.concatenate([x, edge, -edge])
    ours = O.to_lowp(x, dt)
    ref = torch.from_numpy(x).to(tdt).view(torch.int16).numpy().view(np.uint16)
    np.testing.assert_array_equal(ours, ref)


# --------------------------------------------------------------- generator
def test_generator_deterministic_and_in_range():
    a = O.uniform((1000, 37), seed=0)
    b = O.uniform((1000, 37), seed=0)
    c = O.uniform((1000, 37), seed=1)
    np.testing.assert_array_equal(a, b)
    assert not np.array_equal(a, c)
    assert a.min() >= -1.0 and a.max() < 1.0
    assert abs(a.mean()) < 0.02
    # element i only depends on (seed, i): a prefix of a longer draw is identical
    np.testing.assert_array_equal(O.uniform(500, seed=3), O.uniform(1000, seed=3)[:500])


def test_normal_moments():
    z = O.normal(1_000_001, seed=5, mean=0.0, std=1.0)
    assert abs(z.mean()) < 5e-3 and abs(z.std() - 1.0) < 5e-3
    w = O.normal(100_000, seed=6, std=0.02)
    assert abs(w.std() - 0.02) < 1e-3


# --------------------------------------------------------------- restated math
@pytest.mark.parametrize("tA,tB", [(False, False), (True, False), (False, True), (True, True)])
def test_gemm_f32_against_numpy(tA, tB):
    M, N, K = 37, 53, 71
    A = O.uniform((K, M) if tA else (M, K), seed=11)
    B = O.uniform((N, K) if tB else (K, N), seed=12)
    C0 = O.uniform((M, N), seed=13)
    R = 0.75 * ((A.T if tA else A).astype(np.float64) @ (B.T if tB else B).astype(np.float64)) + 0.5 * C0
    C = O.gemm_f32(A, B, C0, transA=tA, transB=tB, alpha=0.75, beta=0.5)
    assert O.rel_frobenius(C, R) <= 1e-5 * np.sqrt(K)


def test_gemm_f32_thread_count_invariant():
    A = O.uniform((64, 200), seed=1)
    B = O.uniform((200, 48), seed=2)
    np.testing.assert_array_equal(O.gemm_f32(A, B, nthreads=1), O.gemm_f32(A, B, nthreads=4))


def test_gemm_f32_sum_order_is_fma_chain():
    """Each output is fma(a_k, b_k, acc) for k ascending — checked against a
    scalar Python loop with math.fma-equivalent float32 steps."""
    A = O.uniform((3, 29), seed=21)
    B = O.uniform((29, 5), seed=22)
    C = O.gemm_f32(A, B)
    for i in range(3):
        for j in range(5):
            acc = np.float32(0)
            for k in range(29):
                acc = np.float32(np.float64(A[i, k]) * np.float64(B[k, j]) + np.float64(acc))
            assert C[i, j] == acc


def test_gemm_f64_against_numpy():
    A = np.asarray(O.uniform((20, 30), seed=3), np.float64)
    B = np.asarray(O.uniform((30, 10), seed=4), np.float64)
    np.testing.assert_allclose(O.gemm_f64(A, B), A @ B, rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("dt", [O.F16, O.BF16])
def test_gemm_lowp_against_numpy(dt):
    M, N, K = 40, 33, 128
    A = O.to_lowp(O.normal((M, K), seed=1) / np.sqrt(K), dt)
    B = O.to_lowp(O.normal((K, N), seed=2), dt)
    R = O.from_lowp(A, dt).astype(np.float64) @ O.from_lowp(B, dt).astype(np.float64)
    C = O.from_lowp(O.gemm_lowp(dt, A, B), dt)
    assert O.max_relative(C, R) <= 1e-2


@pytest.mark.parametrize("trans", [False, True])
def test_gemv_f32_against_numpy(trans):
    M, N = 300, 170
    A = O.uniform((N, M) if trans else (M, N), seed=8)
    x = O.uniform(N, seed=9)
    y0 = O.uniform(M, seed=10)
    R = 2.0 * ((A.T if trans else A).astype(np.float64) @ x.astype(np.float64)) - 1.5 * y0
    y = O.gemv_f32(A, x, y0, trans=trans, alpha=2.0, beta=-1.5)
    assert O.rel_frobenius(y, R) <= 1e-5 * np.sqrt(N)
    np.testing.assert_allclose(O.gemv_f64acc(A, x, trans=trans), (A.T if trans else A).astype(np.float64) @ x,
                               rtol=1e-12, atol=1e-9)


def test_gemm_sample_matches_full():
    A = O.uniform((50, 60), seed=1)
    B = O.uniform((60, 70), seed=2)
    full = A.astype(np.float64) @ B.astype(np.float64)
    rows, cols = np.array([0, 7, 49]), np.array([3, 69])
    np.testing.assert_allclose(O.gemm_sample_f64(A, B, rows, cols), full[np.ix_(rows, cols)], rtol=1e-12)


def test_gemm_rows_cols_matches_the_per_element_sampler():
    """The blocked fp64 rows/columns helper against the C per-element fp64
    sampler (ascending-k sums) on complete rows and columns, with blocks
    smaller than the matrix so the block edges are covered."""
    A = O.uniform((70, 300), seed=3)
    B = O.uniform((300, 90), seed=4)
    rows, cols = np.array([0, 5, 69]), np.array([1, 44, 89])
    R, Q = O.gemm_rows_cols_f64(A, B, rows, cols, block=32)
    np.testing.assert_allclose(R, O.gemm_sample_f64(A, B, rows, np.arange(90)), rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(Q, O.gemm_sample_f64(A, B, np.arange(70), cols), rtol=1e-12, atol=1e-12)
