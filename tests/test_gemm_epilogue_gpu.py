"""Fused GEMM epilogue (cuopx_gemm_ex): C = act(alpha*op(A)op(B) + beta*C + bias).

The operator it replaces is MatMulReluFused<T>::Forward
(src/cuda_op/detail/cuDNN/kernel_fusion.cu:330-370): relu(A*W + bias).
fp32 on the FFMA kernels and fp64 must be BIT-IDENTICAL to the oracle (same
ascending-k fma chain, then the rounded bias add and ReLU), and fp32 also to
the reference's own MatMulReluFused<float>; 3xTF32 within
||C-R||_F/||R||_F <= 1e-5*sqrt(K); fp16/bf16 (1- and 2-SM tcgen05 kernels)
within max|C-R|/max|R| <= 1e-2 of the oracle."""
import numpy as np
import pytest
import torch

import cuop_b200 as cx
import oracle as O
from cuop_b200 import _native as N
from helpers import forced_variant, lowp_bits, to_dev_f32, to_dev_lowp

pytestmark = pytest.mark.gpu
LOWP_TOL = 1e-2
EPIS = [(True, True), (True, False), (False, True)]  # (bias, relu)


@pytest.mark.parametrize("bias,relu", EPIS)
@pytest.mark.parametrize("M,N,K,tA,tB", [(64, 96, 80, False, False), (130, 68, 257, False, False),
                                         (100, 44, 70, True, True), (256, 512, 128, False, False)])
def test_f32_ffma_epilogue_bit_exact(dev, fp32_ffma, M, N, K, tA, tB, bias, relu):
    A = O.uniform((K, M) if tA else (M, K), seed=M)
    B = O.uniform((N, K) if tB else (K, N), seed=N + 1)
    b = O.uniform(N, seed=K + 2) if bias else None
    ref = O.gemm_f32(A, B, transA=tA, transB=tB, bias=b, relu=relu)
    C = cx.gemm(to_dev_f32(A, dev), to_dev_f32(B, dev), transA=tA, transB=tB,
                bias=None if b is None else to_dev_f32(b, dev), relu=relu)
    assert cx.last_kernel().startswith(("gemm_f32_", "gemm_simt_generic")), cx.last_kernel()
    got = C.cpu().numpy()
    assert np.array_equal(got, ref), np.abs(got - ref).max()
    if relu:
        assert (got >= 0).all()


def test_f32_matches_reference_matmul_relu_fused(dev, fp32_ffma):
    """Same inputs through the reference's own MatMulReluFused<float>."""
    if not O.ref_available():
        pytest.skip("reference operators not built")
    M, N, K = 192, 160, 333
    A = O.uniform((M, K), seed=3)
    B = O.uniform((K, N), seed=4)
    b = O.uniform(N, seed=5)
    Ad, Bd, bd = to_dev_f32(A, dev), to_dev_f32(B, dev), to_dev_f32(b, dev)
    ours = cx.gemm(Ad, Bd, bias=bd, relu=True).cpu().numpy()
    Cr = torch.zeros(M, N, device=dev)
    torch.cuda.synchronize()
    assert O.ref_lib().ref_matmul_relu_f32(0, 0, M, N, K, Ad.data_ptr(), Bd.data_ptr(), bd.data_ptr(),
                                           Cr.data_ptr()) == 0
    ref = Cr.cpu().numpy()
    assert np.array_equal(ours, ref), np.abs(ours - ref).max()
    assert np.array_equal(ours, O.gemm_f32(A, B, bias=b, relu=True))


def test_f32_tf32x3_epilogue_within_tolerance(dev):
    M, N, K = 512, 384, 640
    A = O.uniform((M, K), seed=7)
    B = O.uniform((K, N), seed=8)
    b = O.uniform(N, seed=9)
    C = cx.gemm(to_dev_f32(A, dev), to_dev_f32(B, dev), bias=to_dev_f32(b, dev), relu=True)
    assert cx.last_kernel().startswith("gemm_tf32x3_"), cx.last_kernel()
    exact = np.maximum(A.astype(np.float64) @ B.astype(np.float64) + b, 0.0)
    assert O.rel_frobenius(C.cpu().numpy(), exact) <= 0.1 * 1e-5 * np.sqrt(K)


def test_f64_epilogue_bit_exact(dev):
    M, N, K = 70, 50, 90
    A = O.uniform((M, K), seed=1).astype(np.float64)
    B = O.uniform((K, N), seed=2).astype(np.float64)
    b = O.uniform(N, seed=3).astype(np.float64)
    C = cx.gemm(torch.from_numpy(A).to(dev), torch.from_numpy(B).to(dev), bias=torch.from_numpy(b).to(dev),
                relu=True, alpha=0.5)
    ref = O.gemm_f64(A, B, alpha=0.5, bias=b, relu=True)
    assert np.array_equal(C.cpu().numpy(), ref)


@pytest.mark.parametrize("dt", [O.F16, O.BF16])
@pytest.mark.parametrize("bias,relu", EPIS)
@pytest.mark.parametrize("M,N,K,kernel", [(320, 200, 256, "gemm_tc_"), (4096, 2560, 512, "gemm_tc2_256x256"),
                                           (4096, 2600, 512, "gemm_tc2_256x512")])
def test_lowp_epilogue_vs_oracle(dev, dt, M, N, K, kernel, bias, relu):
    A = O.to_lowp(O.normal((M, K), seed=M) / np.sqrt(K), dt)
    B = O.to_lowp(O.normal((K, N), seed=N), dt)
    b = O.to_lowp(O.normal(N, seed=K), dt) if bias else None
    C0 = O.to_lowp(O.normal((M, N), seed=11), dt)
    Cd = to_dev_lowp(C0, dt, dev)
    with forced_variant({"gemm_tc2_256x256": "tc2", "gemm_tc2_256x512": "tc2_256x512"}.get(kernel)):
        cx.gemm(to_dev_lowp(A, dt, dev), to_dev_lowp(B, dt, dev), Cd, alpha=1.25, beta=0.5,
                bias=None if b is None else to_dev_lowp(b, dt, dev), relu=relu)
    assert cx.last_kernel().startswith(kernel), cx.last_kernel()
    rows = np.arange(M) if M <= 512 else np.array([0, 1, 255, 256, 2047, M - 1])
    ref = O.gemm_lowp(dt, A[rows], B, C0[rows], alpha=1.25, beta=0.5, bias=b, relu=relu)
    got = O.from_lowp(lowp_bits(Cd[torch.as_tensor(rows, device=dev)]), dt)
    assert O.max_relative(got, O.from_lowp(ref, dt)) <= LOWP_TOL
    if relu:
        assert (got >= 0).all()


def test_epilogue_argument_checks(dev):
    A = torch.randn(64, 64, device=dev)
    C = torch.empty(64, 64, device=dev)
    lib = N.lib()
    s = torch.cuda.current_stream().cuda_stream
    rc = lib.cuopx_gemm_ex(N.F32, 0, 0, 64, 64, 64, 1.0, A.data_ptr(), 64, A.data_ptr(), 64, 0.0, C.data_ptr(), 64,
                           0, N.EPI_BIAS, s)
    assert rc == N.INVALID_ARGUMENT  # bias flag without a bias vector
    rc = lib.cuopx_gemm_ex(N.F32, 0, 0, 64, 64, 64, 1.0, A.data_ptr(), 64, A.data_ptr(), 64, 0.0, C.data_ptr(), 64,
                           0, 7, s)
    assert rc == N.INVALID_ARGUMENT  # unknown epilogue bits
    rc = lib.cuopx_gemm_ex(N.F32, 0, 0, 64, 64, 64, 1.0, A.data_ptr(), 64, A.data_ptr(), 64, 0.0, C.data_ptr(), 64,
                           C.data_ptr(), N.EPI_BIAS, s)
    assert rc == N.INVALID_ARGUMENT  # bias inside C
