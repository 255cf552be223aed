"""Peer memory across the ranks of one node and the fused column-sharded GEMM.

One process per GPU.  A `SymmetricBuffer` is one allocation of the same size
on every rank (cuopx_peer_alloc), whose IPC handles are exchanged through
torch.distributed so that each rank holds a pointer to every rank's copy
(its own, plus peer mappings over NVLink from cuopx_peer_open).

`PeerShardedGemm` computes Y = X @ W with W split by column blocks over the
ranks and leaves the full Y on every rank without a collective library call:
the GEMM epilogue of rank r stores each finished output tile into column
block r of every rank's output buffer (cuopx_gemm_allgather), between two
cross-GPU barriers (cuopx_peer_barrier).  Peer pointers never pass through
torch: only the local copy is exposed as a tensor.
"""
from __future__ import annotations

import ctypes as C
from typing import Callable, List, Optional

import torch
import torch.distributed as dist

from . import _native as N
from . import ops

_TYPESTR = {torch.float16: "<f2", torch.bfloat16: "<i2", torch.float32: "<f4", torch.uint8: "|u1",
            torch.int32: "<i4"}


def _alloc(nbytes: int):
    ptr = C.c_void_p()
    handle = (C.c_ubyte * N.PEER_HANDLE_BYTES)()
    N.check(N.lib().cuopx_peer_alloc(nbytes, C.byref(ptr), handle), "cuopx_peer_alloc")
    return ptr.value, bytes(handle)


def _open(handle: bytes) -> int:
    ptr = C.c_void_p()
    buf = (C.c_ubyte * N.PEER_HANDLE_BYTES).from_buffer_copy(handle)
    N.check(N.lib().cuopx_peer_open(buf, C.byref(ptr)), "cuopx_peer_open")
    return ptr.value


def _exchange(obj, world: int, group) -> list:
    if world == 1:
        return [obj]
    out = [None] * world
    dist.all_gather_object(out, obj, group=group)
    return out


class _ArrayView:
    """__cuda_array_interface__ over a raw device pointer (local memory only)."""

    def __init__(self, ptr: int, shape, dtype: torch.dtype, owner):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": _TYPESTR[dtype],
                                         "data": (ptr, False), "version": 3, "strides": None}
        self._owner = owner  # keeps the allocation alive while a view exists


class SymmetricBuffer:
    """`nbytes` on every rank; `ptrs[r]` is rank r's copy as seen from this process.

    alloc_fn / open_fn / close_fn / free_fn / exchange_fn default to the
    library's IPC calls and torch.distributed; tests of the host logic on
    CPU ranks substitute fakes.
    """

    def __init__(self, nbytes: int, rank: int, world: int, group=None, *,
                 alloc_fn: Optional[Callable] = None, open_fn: Optional[Callable] = None,
                 close_fn: Optional[Callable] = None, free_fn: Optional[Callable] = None,
                 exchange_fn: Optional[Callable] = None):
        if nbytes <= 0 or not (0 <= rank < world):
            raise ValueError(f"bad symmetric buffer: {nbytes} bytes, rank {rank} of {world}")
        self.nbytes, self.rank, self.world = nbytes, rank, world
        self._close = close_fn or (lambda p: N.check(N.lib().cuopx_peer_close(p), "cuopx_peer_close"))
        self._free = free_fn or (lambda p: N.check(N.lib().cuopx_peer_free(p), "cuopx_peer_free"))
        self.local_ptr, handle = (alloc_fn or _alloc)(nbytes)
        self.ptrs: List[int] = []
        self._opened: List[int] = []
        opener = open_fn or _open
        try:
            handles = (exchange_fn or (lambda h: _exchange(h, world, group)))(handle)
            if len(handles) != world:
                raise RuntimeError(f"handle exchange returned {len(handles)} entries for {world} ranks")
            for r in range(world):
                if r == rank:
                    self.ptrs.append(self.local_ptr)
                else:
                    p = opener(handles[r])
                    self._opened.append(p)
                    self.ptrs.append(p)
        except Exception:
            self.close()
            raise
        self._ptr_array = (C.c_void_p * world)(*self.ptrs)

    def pointer_array(self):
        return self._ptr_array

    def local_tensor(self, shape, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
        """Local copy as a tensor view (no copy; valid while this buffer lives)."""
        numel = 1
        for s in shape:
            numel *= int(s)
        esize = torch.empty((), dtype=dtype).element_size()
        if numel * esize > self.nbytes:
            raise ValueError("view larger than the buffer")
        t = torch.as_tensor(_ArrayView(self.local_ptr, shape, dtype, self), device=device)
        return t.view(torch.bfloat16) if dtype == torch.bfloat16 else t

    def unmap_peers(self) -> None:
        for p in self._opened:
            self._close(p)
        self._opened = []
        self.ptrs = [self.local_ptr if r == self.rank else 0 for r in range(self.world)]
        self._ptr_array = (C.c_void_p * self.world)(*self.ptrs)

    def free_local(self) -> None:
        if self.local_ptr:
            self._free(self.local_ptr)
            self.local_ptr = 0

    def close(self, barrier: Optional[Callable[[], None]] = None) -> None:
        """Unmap the peers' copies, wait for the other ranks to do the same
        (`barrier`), then free the local copy."""
        self.unmap_peers()
        if barrier is not None:
            barrier()
        self.free_local()


def peer_barrier(signals: SymmetricBuffer, stream=None) -> None:
    rc = N.lib().cuopx_peer_barrier(signals.pointer_array(), signals.world, signals.rank, ops._stream(stream))
    N.check(rc, "cuopx_peer_barrier")


class PeerShardedGemm:
    """Y = X @ W, W column-sharded over `world` ranks, full Y left on every rank.

    w_local is this rank's contiguous [K, N/G] block.  The output lives in a
    symmetric buffer of `max_rows` x N; forward() returns the local [M, N]
    view of it, which the next forward() overwrites.
    """

    def __init__(self, w_local: torch.Tensor, rank: int, world: int, max_rows: int, group=None):
        if w_local.dim() != 2 or w_local.dtype not in (torch.float16, torch.bfloat16):
            raise N.CuopError(N.UNSUPPORTED_TYPE, "PeerShardedGemm takes a 2-D fp16/bf16 weight block")
        ops._require_cuda(w_local)
        self.w_local, self.rank, self.world, self.max_rows, self.group = w_local, rank, world, max_rows, group
        self.last_kernel = ""
        self.nb = w_local.size(1)
        self.n_total = world * self.nb
        es = w_local.element_size()
        self.out = SymmetricBuffer(max_rows * self.n_total * es, rank, world, group)
        self.signals = SymmetricBuffer(N.PEER_SIGNAL_BYTES, rank, world, group)
        torch.cuda.synchronize()
        if world > 1:
            # Every rank has mapped every buffer and finished its set-up before
            # any barrier kernel can start waiting for it.
            dist.barrier(group=group)

    def forward(self, X: torch.Tensor, stream=None) -> torch.Tensor:
        M, K = X.shape
        if M > self.max_rows or K != self.w_local.size(0) or X.dtype != self.w_local.dtype:
            raise N.CuopError(N.SHAPE_MISMATCH, f"X {tuple(X.shape)} {X.dtype} vs W block "
                                                f"{tuple(self.w_local.shape)}, max rows {self.max_rows}")
        s = ops._stream(stream)
        peer_barrier(self.signals, s)  # peers are done reading their previous outputs
        rc = N.lib().cuopx_gemm_allgather(ops._dtype_code(X), 0, 0, M, self.nb, K, 1.0, X.data_ptr(), ops._row_ld(X),
                                          self.w_local.data_ptr(), ops._row_ld(self.w_local),
                                          self.out.pointer_array(), self.world, self.rank, self.n_total, s)
        N.check(rc, "cuopx_gemm_allgather")
        self.last_kernel = ops.last_kernel()  # the GEMM variant (before the barrier's launch)
        peer_barrier(self.signals, s)  # every rank's block has landed here
        return self.out.local_tensor((M, self.n_total), X.dtype, X.device)

    def close(self) -> None:
        """Collective: every rank calls it (no rank frees memory a peer still maps)."""
        torch.cuda.synchronize()
        self.out.unmap_peers()
        self.signals.unmap_peers()
        if self.world > 1:
            dist.barrier(group=self.group)
        self.out.free_local()
        self.signals.free_local()
