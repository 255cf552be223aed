"""Fused column-sharded GEMM + all-gather (cuopx_gemm_allgather) on one GPU.

Several ranks are emulated in one process: their full outputs are local
buffers, and rank r's call writes its column block into all of them (the
peer stores go to local memory here; over NVLink in the multi-GPU test).
The barrier is only run with world 1, or against a flag nothing sets (its
bounded wait must run out and report CUOPX_DEVERR_PEER_TIMEOUT): barrier
kernels that wait on each other never run as separate launches on one GPU.
Tolerance: fp16/bf16 max|C-R|/max|R| <= 1e-2 against the oracle."""
import ctypes as C

import numpy as np
import pytest
import torch

import cuop_b200 as cx
import oracle as O
from cuop_b200 import _native as N
from cuop_b200 import peer
from helpers import forced_variant, fp32_reference_gpu, lowp_bits, to_dev_lowp

pytestmark = pytest.mark.gpu
LOWP_TOL = 1e-2
TDT = {O.F16: torch.float16, O.BF16: torch.bfloat16}


def _call(dt, M, nb, K, A, Wb, outs, rank, tA=False, tB=False, alpha=1.0):
    world = len(outs)
    arr = (C.c_void_p * world)(*[o.data_ptr() for o in outs])
    lda = A.stride(0)
    ldb = Wb.stride(0)
    stream = torch.cuda.current_stream().cuda_stream
    return N.lib().cuopx_gemm_allgather(dt, int(tA), int(tB), M, nb, K, alpha, A.data_ptr(), lda, Wb.data_ptr(), ldb,
                                        arr, world, rank, world * nb, stream)


CASES = [  # (world, M, nb, K, tA, tB)
    (2, 1024, 512, 512, False, False),
    (3, 300, 264, 320, False, False),
    (4, 512, 256, 256, True, False),
    (2, 640, 384, 288, False, True),
    (8, 256, 256, 256, False, False),
]


PATHS = [("tc2", "gemm_tc2_256x256"), ("tc2_256x512", "gemm_tc2_256x512"), ("tc_128x128", "gemm_tc_128x128"),
         ("tc_128x256", "gemm_tc_128x256"), ("tc2_256x128", "gemm_tc2_256x128")]


@pytest.mark.parametrize("variant,kernel", PATHS)
@pytest.mark.parametrize("dt", [O.F16, O.BF16])
@pytest.mark.parametrize("world,M,nb,K,tA,tB", CASES)
def test_allgather_every_rank_gets_every_block(dev, dt, world, M, nb, K, tA, tB, variant, kernel):
    A = O.to_lowp(O.normal((K, M) if tA else (M, K), seed=M + K) / np.sqrt(K), dt)
    W = O.to_lowp(O.normal((world * nb, K) if tB else (K, world * nb), seed=nb + 3), dt)
    Ad = to_dev_lowp(A, dt, dev)
    Wd = to_dev_lowp(W, dt, dev)
    outs = [torch.full((M, world * nb), float("nan"), dtype=TDT[dt], device=dev) for _ in range(world)]
    for r in range(world):
        Wb = (Wd[r * nb:(r + 1) * nb] if tB else Wd[:, r * nb:(r + 1) * nb]).contiguous()
        with forced_variant(variant):
            assert _call(dt, M, nb, K, Ad, Wb, outs, r, tA, tB, alpha=1.25) == 0
        # The 1-SM peer path is compiled for the row-major layout only;
        # transposed operands take the 2-SM kernel's peer path.
        expect = kernel if not (tA or tB) or kernel.startswith("gemm_tc2") else "gemm_tc2_256x256"
        assert cx.last_kernel() == expect + ("_peer" if world > 1 else "")
    torch.cuda.synchronize()
    for o in outs[1:]:  # every rank's copy is the same bits
        assert torch.equal(o.view(torch.int16), outs[0].view(torch.int16))
    full = 1.25 * fp32_reference_gpu(Ad, Wd, tA, tB)
    assert not torch.isnan(outs[0].float()).any()
    assert O.max_relative(outs[0].float().cpu().numpy(), full.cpu().numpy()) <= LOWP_TOL
    rows = np.array([0, M // 2, M - 1])
    ref = O.gemm_lowp(dt, A[:, rows] if tA else A[rows], W, transA=tA, transB=tB, alpha=1.25)
    got = O.from_lowp(lowp_bits(outs[world - 1][torch.as_tensor(rows, device=dev)]), dt)
    assert O.max_relative(got, O.from_lowp(ref, dt)) <= LOWP_TOL


def test_allgather_uses_pair_tiles_by_default(dev):
    """Pair tiles at any rank count unless a 1-SM path is forced."""
    for world, nb, K in ((2, 4096, 4096), (8, 256, 2048)):
        A = torch.randn(2048, K, device=dev).half()
        Wb = torch.randn(K, nb, device=dev).half()
        outs = [torch.empty(2048, world * nb, device=dev, dtype=torch.half) for _ in range(world)]
        assert _call(O.F16, 2048, nb, K, A, Wb, outs, 0) == 0
        assert cx.last_kernel() == "gemm_tc2_256x256_peer", (world, cx.last_kernel())


def test_allgather_touches_only_its_block(dev):
    dt, world, M, nb, K = O.BF16, 3, 520, 264, 256
    A = torch.randn(M, K, device=dev).bfloat16()
    Wb = torch.randn(K, nb, device=dev).bfloat16()
    outs = [torch.full((M, world * nb), 7.0, dtype=torch.bfloat16, device=dev) for _ in range(world)]
    assert _call(dt, M, nb, K, A, Wb, outs, 1) == 0
    torch.cuda.synchronize()
    ref = fp32_reference_gpu(A, Wb)
    for o in outs:
        assert (o[:, :nb] == 7.0).all() and (o[:, 2 * nb:] == 7.0).all()
        assert O.max_relative(o[:, nb:2 * nb].float().cpu().numpy(), ref.cpu().numpy()) <= LOWP_TOL


def test_allgather_rejects_and_declines(dev):
    A = torch.randn(512, 512, device=dev).half()
    Wb = torch.randn(512, 256, device=dev).half()
    outs = [torch.empty(512, 512, device=dev, dtype=torch.half) for _ in range(2)]
    assert _call(O.F16, 512, 256, 512, A, Wb, outs, 2) == N.INVALID_ARGUMENT  # rank out of range
    small = [torch.empty(128, 256, device=dev, dtype=torch.half) for _ in range(2)]
    assert _call(O.F16, 128, 128, 512, A[:128], Wb[:, :128].contiguous(), small, 0) == N.NOT_IMPLEMENTED
    a32 = torch.randn(512, 512, device=dev)
    w32 = torch.randn(512, 256, device=dev)
    o32 = [torch.empty(512, 512, device=dev) for _ in range(2)]
    assert _call(N.F32, 512, 256, 512, a32, w32, o32, 0) == N.NOT_IMPLEMENTED


def test_peer_sharded_gemm_world1(dev):
    X = (torch.randn(1024, 512, device=dev) / 23).half()
    W = torch.randn(512, 768, device=dev).half()
    sg = peer.PeerShardedGemm(W, rank=0, world=1, max_rows=2048)
    try:
        Y = sg.forward(X)
        assert Y.shape == (1024, 768) and Y.dtype == torch.half and Y.device == X.device
        ref = fp32_reference_gpu(X, W)
        assert O.max_relative(Y.float().cpu().numpy(), ref.cpu().numpy()) <= LOWP_TOL
        first = Y.clone()
        Y2 = sg.forward(X[:512])  # fewer rows, same buffer
        assert Y2.data_ptr() == Y.data_ptr()
        assert torch.equal(Y2, first[:512])
    finally:
        sg.close()


def test_peer_barrier_times_out_on_a_missing_rank(dev):
    """Rank 1 never arrives: the bounded wait gives up (about 5 s) and records
    the timeout code; the context stays usable."""
    sig = [torch.zeros(N.PEER_SIGNAL_BYTES // 4, dtype=torch.int32, device=dev) for _ in range(2)]
    arr = (C.c_void_p * 2)(*[s.data_ptr() for s in sig])
    cx.clear_device_error()
    assert N.lib().cuopx_peer_barrier(arr, 2, 0, torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    code = cx.device_error()
    cx.clear_device_error()
    assert code == N.DEVERR_PEER_TIMEOUT
    assert sig[0][0].item() == 1 and sig[1][0].item() == 1 and sig[0][1].item() == 0
    x = torch.ones(4, device=dev)
    assert float(cx.asum(x).item()) == 4.0  # context still works


def test_peer_barrier_world1_counts_epochs(dev):
    sig = torch.zeros(N.PEER_SIGNAL_BYTES // 4, dtype=torch.int32, device=dev)
    arr = (C.c_void_p * 1)(sig.data_ptr())
    for _ in range(3):
        assert N.lib().cuopx_peer_barrier(arr, 1, 0, torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    assert sig[0].item() == 3 and sig[64].item() == 3
