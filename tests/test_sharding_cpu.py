"""Multi-GPU host logic on CPU ranks (gloo, world_size 2): shard ranges, the
chunked all-gather + column-block gather of ColumnShardedGemm, and batch
sharding.  The GEMM and gather kernels are replaced by torch CPU equivalents
here; the CUDA kernels themselves are covered by the -m gpu tests."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cuop_b200.sharding import ColumnShardedGemm, shard_range, split_columns


def test_shard_range_covers_exactly():
    for total in (0, 1, 7, 4096, 28672, 4097):
        for world in (1, 2, 3, 8):
            spans = [shard_range(total, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [e - s for s, e in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(10, 2, 2)


def _cpu_gemm(X, W, out=None):
    if out is None:
        return X @ W
    out.copy_(X @ W)
    return out


def _cpu_gather(blocks, out):
    G, M, nb = blocks.shape
    out.copy_(blocks.permute(1, 0, 2).reshape(M, G * nb))
    return out


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(0)
        M, K, N = 37, 24, 16
        X = torch.randn(M, K, generator=g, dtype=torch.float64)
        W = torch.randn(K, N, generator=g, dtype=torch.float64)
        Wl = split_columns(W, rank, world)
        sg = ColumnShardedGemm(Wl, world, chunks=3, gemm_fn=_cpu_gemm, gather_fn=_cpu_gather)
        Y = sg.forward(X)
        ok_full = torch.allclose(Y, X @ W, rtol=0, atol=1e-12)
        ok_local = torch.allclose(sg.forward(X, gather=False), X @ Wl, rtol=0, atol=1e-12)
        # batch sharding: every batch computed by exactly one rank, no collective needed
        b0, b1 = shard_range(10, rank, world)
        counts = torch.zeros(10, dtype=torch.int64)
        counts[b0:b1] += 1
        dist.all_reduce(counts)
        results[rank] = (bool(ok_full), bool(ok_local), counts.tolist())
    finally:
        dist.destroy_process_group()


def test_column_sharded_gather_and_batch_sharding_two_ranks():
    world = 2
    mgr = mp.get_context("spawn").Manager()
    results = mgr.dict()
    mp.start_processes(_worker, args=(world, _free_port(), results), nprocs=world, join=True, start_method="spawn")
    for r in range(world):
        ok_full, ok_local, counts = results[r]
        assert ok_full and ok_local
        assert counts == [1] * 10


def _absent_rank_worker(rank, world, port, results):
    """Rank 1 initialises the group and then never joins the all-gather
    (it stays alive past rank 0's timeout); rank 0 must get a
    CollectiveError after the group's 2 s timeout, not hang."""
    import datetime
    import time

    from cuop_b200.sharding import CollectiveError

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=2))
    try:
        if rank == 1:
            time.sleep(8)
            results[rank] = "absent"
            return
        g = torch.Generator().manual_seed(0)
        X = torch.randn(8, 4, generator=g, dtype=torch.float64)
        Wl = torch.randn(4, 3, generator=g, dtype=torch.float64)
        sg = ColumnShardedGemm(Wl, world, chunks=2, gemm_fn=_cpu_gemm, gather_fn=_cpu_gather)
        t0 = time.monotonic()
        try:
            sg.forward(X)
            results[rank] = ("no error", time.monotonic() - t0, 0)
        except CollectiveError as e:
            results[rank] = ("CollectiveError", time.monotonic() - t0, e.status)
    finally:
        dist.destroy_process_group()


def test_column_sharded_gather_reports_a_rank_that_never_joins():
    world = 2
    mgr = mp.get_context("spawn").Manager()
    results = mgr.dict()
    mp.start_processes(_absent_rank_worker, args=(world, _free_port(), results), nprocs=world, join=True,
                       start_method="spawn")
    kind, elapsed, status = results[0]
    assert kind == "CollectiveError" and status == 1003
    assert elapsed < 30
    assert results[1] == "absent"
