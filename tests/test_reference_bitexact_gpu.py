"""FFMA mode against the reference's own fp32 operators, bit for bit.

oracle/_ref/libcuop_ref.so is the reference's Gemm<float> and Gemv<float>
compiled from its sources (oracle/Makefile); each call goes through its
public operator API (SetWeight + Forward).  With cuopx_set_fp32_gemm_mode
(FP32_FFMA), our GEMM and GEMV must return exactly the same bits:

* GEMM, untransposed operands, on every kernel the reference's selector
  picks (src/cuda_op/detail/cuBlas/gemm.cu:305-356): gemm_kernel_basic (small),
  gemm_kernel_tiled, gemm_kernel_warp_optimized and gemm_kernel_blocked (C1
  1024^3).  All accumulate one fma chain over k in ascending order and end
  with `alpha * sum + beta * C` (gemm.cu:41), which nvcc builds as
  fma(alpha, sum, beta*C); alpha and beta are chosen so that every other
  epilogue form would differ in the last bit (0.7 and 1.3, not powers of two).
* GEMV through gemv_kernel (gemv.cu:10-23; the reference uses it when M or N
  is below 64) in both layouts, and the transposed layout of
  gemv_kernel_tiled_vectorized (M, N >= 1024), whose chain is also ascending.

Not compared here, because the reference's own kernels differ from their
stated math or cannot run: transposed GEMM (the reference's selector sends
transposes to kernels that ignore the flags, gemm.cu:315-324), the
untransposed GEMV for M, N >= 64 (float4 partial sums in a different order),
and Gemv<float> with 256 <= M, N where M or N is below 1024: its
gemv_kernel_shared<T,128> runs with 256 threads and indexes its 128-element
shared array with the thread index (gemv.cu:25-45, launched at gemv.cu:232-236),
an out-of-bounds access that faulted on a B200.
"""
import numpy as np
import pytest
import torch

import cuop_b200 as cx
import oracle as O
from helpers import to_dev_f32

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not O.ref_available(), reason="reference operators not built (oracle/Makefile ref)")]

ALPHA_BETA = [(1.0, 0.0), (0.7, 1.3), (-1.5, 0.25)]

# (M, N, K, kernel the reference's selector picks)
GEMM_CASES = [
    (1, 1, 1, "basic"), (37, 45, 29, "basic"), (100, 70, 50, "basic"),
    (200, 150, 130, "tiled"), (300, 200, 100, "tiled"),
    (512, 512, 512, "warp_optimized"), (600, 300, 520, "warp_optimized"),
    (1024, 1024, 1024, "blocked"),
]


def _ref_gemm(A, B, C0, alpha, beta, dev):
    M, K = A.shape
    N = B.shape[1]
    dA, dB, dC = to_dev_f32(A, dev), to_dev_f32(B, dev), to_dev_f32(C0, dev)
    torch.cuda.synchronize()
    rc = O.ref_lib().ref_gemm_f32(0, 0, M, N, K, float(np.float32(alpha)), dA.data_ptr(), dB.data_ptr(),
                                  float(np.float32(beta)), dC.data_ptr())
    assert rc == 0
    return dC.cpu().numpy()


@pytest.mark.parametrize("alpha,beta", ALPHA_BETA)
@pytest.mark.parametrize("M,N,K,kernel", GEMM_CASES)
def test_gemm_ffma_equals_reference_operator(dev, fp32_ffma, M, N, K, kernel, alpha, beta):
    A = O.uniform((M, K), seed=M + 11)
    B = O.uniform((K, N), seed=N + 12)
    C0 = O.uniform((M, N), seed=K + 13)
    ref = _ref_gemm(A, B, C0, alpha, beta, dev)
    ours = cx.gemm(to_dev_f32(A, dev), to_dev_f32(B, dev), to_dev_f32(C0, dev), alpha=float(np.float32(alpha)),
                   beta=float(np.float32(beta))).cpu().numpy()
    assert cx.last_kernel().startswith("gemm_f32_") or cx.last_kernel() == "gemm_simt_generic", cx.last_kernel()
    np.testing.assert_array_equal(ours, ref, err_msg=f"reference kernel {kernel}, ours {cx.last_kernel()}")
    # The oracle's restatement is pinned to the same bits.
    np.testing.assert_array_equal(O.gemm_f32(A, B, C0, alpha=float(np.float32(alpha)),
                                             beta=float(np.float32(beta))), ref)


def test_c1_default_mode_within_tolerance_of_reference(dev):
    """C1 in the default mode (3xTF32) against the reference operator:
    within the fp32 bound, and not silently TF32 (far inside it)."""
    n = 1024
    A, B = O.uniform((n, n), seed=0), O.uniform((n, n), seed=1)
    ref = _ref_gemm(A, B, np.zeros((n, n), np.float32), 1.0, 0.0, dev)
    ours = cx.gemm(to_dev_f32(A, dev), to_dev_f32(B, dev)).cpu().numpy()
    assert cx.last_kernel().startswith("gemm_tf32x3"), cx.last_kernel()
    assert O.rel_frobenius(ours, ref) <= 0.1 * 1e-5 * np.sqrt(n)


# (M, N, trans): gemv_kernel when M or N < 64; the transposed tiled kernel at >= 1024.
GEMV_CASES = [
    (1, 1, False), (50, 40, False), (50, 40, True), (60, 33, True), (2000, 40, False), (2000, 40, True),
    (40, 3000, False), (40, 3000, True), (1024, 2048, True), (8192, 8192, True),
]


@pytest.mark.parametrize("alpha,beta", ALPHA_BETA)
@pytest.mark.parametrize("M,N,trans", GEMV_CASES)
def test_gemv_ffma_equals_reference_operator(dev, fp32_ffma, M, N, trans, alpha, beta):
    if trans is False and min(M, N) >= 64:
        pytest.fail("untransposed GEMV with M, N >= 64 is not the reference's gemv_kernel")
    assert not (256 <= M and 256 <= N and (M < 1024 or N < 1024)), "reference Gemv faults in this range"
    A = O.uniform((N, M) if trans else (M, N), seed=M + 21)  # transposed: the buffer is read as A[col*M+row]
    x = O.uniform(N, seed=22)
    y0 = O.uniform(M, seed=23)
    a32, b32 = float(np.float32(alpha)), float(np.float32(beta))
    dA, dx, dy = to_dev_f32(A, dev), to_dev_f32(x, dev), to_dev_f32(y0, dev)
    torch.cuda.synchronize()
    assert O.ref_lib().ref_gemv_f32(int(trans), M, N, a32, dA.data_ptr(), dx.data_ptr(), b32, dy.data_ptr()) == 0
    ref = dy.cpu().numpy()
    ours = cx.gemv(dA, dx, to_dev_f32(y0, dev), trans=trans, alpha=a32, beta=b32).cpu().numpy()
    assert cx.last_kernel() == "gemv_ordered", cx.last_kernel()
    np.testing.assert_array_equal(ours, ref)
    np.testing.assert_array_equal(O.gemv_f32(A, x, y0, trans=trans, alpha=a32, beta=b32), ref)
