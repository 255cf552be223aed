"""Strided batched GEMM parity (BatchMatMul / GemmBatched path)."""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

import cuop_b200 as cx
import oracle as O
from helpers import fp32_reference_gpu, lowp_bits, to_dev_f32, to_dev_lowp

pytestmark = pytest.mark.gpu
GOLD = json.loads((Path(__file__).parent / "golden" / "known_answers.json").read_text())


def test_known_answer_batch3d(dev):
    g = GOLD["matmul_batch3d"]  # test/cuDNN/test_matmul/test_matmul.cpp:41-67
    A = to_dev_f32(np.array(g["A"]).reshape(2, 2, 3), dev)
    B = to_dev_f32(np.array(g["B"]).reshape(2, 3, 4), dev)
    C = cx.batched_gemm(A, B)
    np.testing.assert_allclose(C.cpu().numpy().ravel(), g["expected"], atol=g["tol"])


@pytest.mark.parametrize("batch,M,N,K", [(3, 33, 17, 65), (16, 128, 128, 64), (5, 100, 200, 300)])
def test_f32_bit_exact(dev, fp32_ffma, batch, M, N, K):
    A = O.uniform((batch, M, K), seed=1)
    B = O.uniform((batch, K, N), seed=2)
    C0 = O.uniform((batch, M, N), seed=3)
    ref = O.gemm_batched_f32(A, B, C0, alpha=1.5, beta=0.25)
    C = cx.batched_gemm(to_dev_f32(A, dev), to_dev_f32(B, dev), to_dev_f32(C0, dev), alpha=1.5, beta=0.25)
    np.testing.assert_array_equal(C.cpu().numpy(), ref)


def test_f32_vs_reference_batchmatmul(dev):
    """fp32 analogue of C4 (smaller batch) against the reference's own
    BatchMatMul<float>::Forward compiled from its sources."""
    if not O.ref_available():
        pytest.skip("reference operators not built")
    batch, M, N, K = 256, 128, 128, 64
    A32 = O.normal((batch, M, K), seed=0)
    B32 = O.normal((batch, K, N), seed=1)
    A, B = to_dev_f32(A32, dev), to_dev_f32(B32, dev)
    C = cx.batched_gemm(A, B)
    Cr = torch.zeros(batch, M, N, device=dev)
    torch.cuda.synchronize()
    assert O.ref_lib().ref_batchmatmul_f32(batch, M, N, K, A.data_ptr(), B.data_ptr(), Cr.data_ptr()) == 0
    exact = np.einsum("bmk,bkn->bmn", A32.astype(np.float64), B32.astype(np.float64))
    assert O.rel_frobenius(Cr.cpu().numpy(), exact) <= 1e-5 * np.sqrt(K)
    assert O.rel_frobenius(C.cpu().numpy(), exact) <= 1e-5 * np.sqrt(K)


@pytest.mark.parametrize("dt", [O.F16, O.BF16])
@pytest.mark.parametrize("batch,M,N,K", [(7, 128, 128, 64), (4, 200, 136, 72), (33, 64, 256, 128)])
def test_lowp_tcgen05_vs_oracle(dev, dt, batch, M, N, K):
    A = O.to_lowp(O.normal((batch, M, K), seed=batch), dt)
    B = O.to_lowp(O.normal((batch, K, N), seed=M), dt)
    C0 = O.to_lowp(O.normal((batch, M, N), seed=N), dt)
    ref = O.gemm_batched_lowp(dt, A, B, C0, alpha=0.5, beta=0.5)
    Cd = to_dev_lowp(C0, dt, dev)
    cx.batched_gemm(to_dev_lowp(A, dt, dev), to_dev_lowp(B, dt, dev), Cd, alpha=0.5, beta=0.5)
    assert cx.last_kernel().startswith("gemm_tc_"), cx.last_kernel()
    assert O.max_relative(O.from_lowp(lowp_bits(Cd), dt), O.from_lowp(ref, dt)) <= 1e-2


def test_c4_bf16_batched_full(dev):
    """C4: 4096 x (128x128x64) bf16, inputs N(0,1), fp32 accumulate."""
    batch, M, N, K = 4096, 128, 128, 64
    dt = O.BF16
    A16 = O.to_lowp(O.normal((batch, M, K), seed=0), dt)
    B16 = O.to_lowp(O.normal((batch, K, N), seed=1), dt)
    A, B = to_dev_lowp(A16, dt, dev), to_dev_lowp(B16, dt, dev)
    C = cx.batched_gemm(A, B)
    assert cx.last_kernel() == "gemm_tc_128x128_2cta"
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    full = torch.bmm(A.float(), B.float())
    torch.backends.cuda.matmul.allow_tf32 = prev
    assert O.max_relative(C.float().cpu().numpy(), full.cpu().numpy()) <= 1e-2
    for b in (0, 1, 2047, 4095):  # oracle on sampled batches, bit patterns
        ref = O.gemm_lowp(dt, A16[b], B16[b])
        got = lowp_bits(C[b])
        assert O.max_relative(O.from_lowp(got, dt), O.from_lowp(ref, dt)) <= 1e-2


def test_shared_b_stride_zero(dev, fp32_ffma):
    """strideB == 0 broadcasts one B to every batch (generic path)."""
    from cuop_b200 import _native as N

    batch, M, Nn, K = 6, 40, 24, 16
    A32 = O.uniform((batch, M, K), seed=1)
    B32 = O.uniform((K, Nn), seed=2)
    A, B = to_dev_f32(A32, dev), to_dev_f32(B32, dev)
    C = torch.empty(batch, M, Nn, device=dev)
    rc = N.lib().cuopx_gemm_strided_batched(N.F32, 0, 0, M, Nn, K, 1.0, A.data_ptr(), K, M * K, B.data_ptr(), Nn, 0,
                                            0.0, C.data_ptr(), Nn, M * Nn, batch,
                                            torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    ref = O.gemm_batched_f32(A32, np.broadcast_to(B32, (batch, K, Nn)).copy())
    np.testing.assert_array_equal(C.cpu().numpy(), ref)


@pytest.mark.parametrize("beta", [0.0, 0.5])
def test_batched_gemm_host_streams_pinned_buffers(dev, beta):
    """The host-buffer form (chunks streamed through the GPU, copies in both
    directions overlapped with the GEMMs) returns exactly the device call's
    bits, for a batch that is not a multiple of the chunk, twice in a row
    (the second call reuses the staging buffers)."""
    batch, M, N, K = 1000, 128, 128, 64
    for call in range(2):
        g = torch.Generator().manual_seed(40 + call)
        A = torch.randn(batch, M, K, generator=g).bfloat16().pin_memory()
        B = torch.randn(batch, K, N, generator=g).bfloat16().pin_memory()
        C0 = torch.randn(batch, M, N, generator=g).bfloat16()
        C = C0.clone().pin_memory()
        cx.batched_gemm_host(A, B, C, beta=beta, chunk=96)
        Cd = C0.to(dev)
        cx.batched_gemm(A.to(dev), B.to(dev), Cd, beta=beta)
        torch.cuda.synchronize()
        assert torch.equal(C, Cd.cpu()), call


def test_batched_gemm_host_refuses_device_or_pageable_tensors(dev):
    A = torch.zeros(2, 8, 8, dtype=torch.bfloat16)
    with pytest.raises(cx.CuopError):
        cx.batched_gemm_host(A, A.clone(), A.clone())  # pageable host memory
    with pytest.raises(cx.CuopError):
        cx.batched_gemm_host(A.to(dev), A.to(dev), A.to(dev))
