"""Worker for the multi-GPU peer-store GEMM test (one process per GPU, run by
torch.distributed.run from tests/test_peer_mgpu.py).

Each rank builds the same seeded X [M, K] and W [K, N] on the host, keeps
W's column block, and runs PeerShardedGemm (fused GEMM + all-gather over
NVLink peer stores) and ColumnShardedGemm (GEMM + NCCL all-gather + gather
kernel).  Checks: the full output on every rank is within the fp16/bf16
tolerance (max|C-R|/max|R| <= 1e-2) of an fp32 product, every rank holds the
same bits, and a second forward with new inputs replaces the first."""
import datetime
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import cuop_b200 as cx  # noqa: E402
from cuop_b200 import peer, sharding  # noqa: E402

TOL = 1e-2


def max_rel(got, ref):
    return float((got.float() - ref).abs().max() / ref.abs().max())


def ref_product(X, W):
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        return X.float() @ W.float()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    ok = True
    for dtype, (M, K, nb) in ((torch.float16, (1024, 512, 512)), (torch.bfloat16, (640, 384, 264))):
        g = torch.Generator().manual_seed(5)
        X = (torch.randn(M, K, generator=g) / K ** 0.5).to(dtype).to(dev)
        W = torch.randn(K, world * nb, generator=g).to(dtype).to(dev)
        Wl = sharding.split_columns(W, rank, world)
        ref = ref_product(X, W)
        sg = peer.PeerShardedGemm(Wl, rank, world, max_rows=M)
        Y = sg.forward(X)
        torch.cuda.synchronize()
        err = max_rel(Y, ref)
        ok &= err <= TOL
        ok &= cx.last_kernel() == "peer_barrier"
        bits = Y.view(torch.int16).to(torch.int64).sum().reshape(1)
        allbits = [torch.zeros_like(bits) for _ in range(world)]
        dist.all_gather(allbits, bits)
        ok &= all(int(b.item()) == int(allbits[0].item()) for b in allbits)
        # second call with other inputs: the buffer is reused, results replaced
        X2 = (torch.randn(M, K, generator=g) / K ** 0.5).to(dtype).to(dev)
        Y2 = sg.forward(X2)
        torch.cuda.synchronize()
        err2 = max_rel(Y2, ref_product(X2, W))
        ok &= err2 <= TOL
        # NCCL path on the same problem
        cs = sharding.ColumnShardedGemm(Wl, world)
        Yn = cs.forward(X)
        torch.cuda.synchronize()
        errn = max_rel(Yn, ref)
        ok &= errn <= TOL
        print(f"rank {rank} {dtype} M={M} K={K} nb={nb}: peer err {err:.2e}, second {err2:.2e}, nccl {errn:.2e}",
              flush=True)
        sg.close()
    code = cx.device_error()
    ok &= code == 0
    flag = torch.tensor([1 if ok else 0], device=dev)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    dist.destroy_process_group()
    if rank == 0:
        print("PEER_MGPU", "OK" if flag.item() == 1 else "FAIL", flush=True)
    sys.exit(0 if flag.item() == 1 else 1)


if __name__ == "__main__":
    main()
