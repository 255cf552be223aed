"""Host logic of the peer-memory layer on CPU ranks (gloo, world_size 2):
handle exchange, the per-rank pointer table (own copy at its own index,
peer mappings elsewhere), and the teardown order (unmap peers, barrier, free
the local copy).  Allocation and mapping are fakes here; the real IPC calls
and kernels are covered by the -m gpu tests."""
import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from cuop_b200 import _native as N
from cuop_b200.peer import SymmetricBuffer


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    log = []
    try:
        def alloc(n):
            log.append(("alloc", n))
            return 0x1000 * (rank + 1), bytes([rank]) * N.PEER_HANDLE_BYTES

        def opener(h):
            assert len(h) == N.PEER_HANDLE_BYTES
            log.append(("open", h[0]))
            return 0x100000 + 0x1000 * (h[0] + 1)

        def exchange(h):
            out = [None] * world
            dist.all_gather_object(out, h)
            return out

        buf = SymmetricBuffer(4096, rank, world, alloc_fn=alloc, open_fn=opener,
                              close_fn=lambda p: log.append(("close", p)),
                              free_fn=lambda p: log.append(("free", p)), exchange_fn=exchange)
        ptrs = list(buf.ptrs)
        arr = [buf.pointer_array()[i] for i in range(world)]
        buf.close(barrier=lambda: (log.append(("barrier",)), dist.barrier()))
        results[rank] = (ptrs, arr, log)
    finally:
        dist.destroy_process_group()


def test_symmetric_buffer_pointer_table_and_teardown():
    world = 2
    mgr = mp.get_context("spawn").Manager()
    results = mgr.dict()
    mp.start_processes(_worker, args=(world, _free_port(), results), nprocs=world, start_method="spawn")
    for rank in range(world):
        ptrs, arr, log = results[rank]
        expect = [0x1000 * (r + 1) if r == rank else 0x100000 + 0x1000 * (r + 1) for r in range(world)]
        assert ptrs == expect and arr == expect
        peers = [0x100000 + 0x1000 * (r + 1) for r in range(world) if r != rank]
        assert log[0] == ("alloc", 4096)
        assert log[1:] == [("open", r) for r in range(world) if r != rank] + \
            [("close", p) for p in peers] + [("barrier",), ("free", 0x1000 * (rank + 1))]


def test_symmetric_buffer_rejects_bad_arguments():
    with pytest.raises(ValueError):
        SymmetricBuffer(0, 0, 1, alloc_fn=lambda n: (1, b"x" * 64))
    with pytest.raises(ValueError):
        SymmetricBuffer(64, 2, 2, alloc_fn=lambda n: (1, b"x" * 64))
    with pytest.raises(RuntimeError):
        SymmetricBuffer(64, 0, 2, alloc_fn=lambda n: (1, b"x" * 64), exchange_fn=lambda h: [h],
                        free_fn=lambda p: None)
