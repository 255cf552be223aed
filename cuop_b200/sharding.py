"""Multi-GPU sharding of the GEMM paths (one process per GPU).

The reference is single-GPU; these two strategies are what the batched and
large-GEMM paths need on one 8-GPU box:

* Batch sharding (strided batched GEMM): rank r owns batches
  [r*B/G, (r+1)*B/G) of contiguous A/B/C and runs one local batched call.
  There is no data-path collective.
* Column sharding (large GEMM / linear layer): rank r holds the weight column
  block W[:, r*N/G:(r+1)*N/G] as its own contiguous [K, N/G] matrix and
  computes Y_r = X W_r.  Only when the caller wants the full Y on every rank
  is there an exchange: per M-chunk, an NCCL all-gather of that chunk's
  [rows, N/G] blocks into a [G, rows, N/G] receive buffer, issued right after
  the chunk's GEMM so the transfer of chunk c overlaps the GEMM of chunk c+1,
  then the column-block gather kernel writes those rows of row-major [M, N].

torch.distributed (NCCL over NVLink/NVSwitch) is plumbing only; every GEMM and
the gather run through libcuopx.so.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Optional

import torch
import torch.distributed as dist

from . import _native, ops


class CollectiveError(RuntimeError):
    """A collective of the column-sharded path did not complete: a rank died,
    left, or did not join within the process group's timeout.  `status` is
    cuOP's TIMEOUT StatusCode value.  The process group is unusable after
    it: destroy it and build a new one before the next sharded call.

    This is raised where the backend reports the failure to the caller,
    which is what a gloo process group does (tested with a rank that never
    joins).  An NCCL process group normally does not: its watchdog thread
    notices the timed-out collective and aborts the whole process (torch's
    TORCH_NCCL_ASYNC_ERROR_HANDLING default), so no exception reaches this
    code.  A caller that wants the error on NCCL instead has to turn that
    handling off (TORCH_NCCL_ASYNC_ERROR_HANDLING=0, or 2 to only clean up)
    and then finds hung ranks by their own timeout; this path is not tested
    on NCCL."""

    status = _native.TIMEOUT


def shard_range(total: int, rank: int, world: int) -> tuple[int, int]:
    """Balanced contiguous split: the first (total % world) ranks get one extra."""
    if world <= 0 or not (0 <= rank < world):
        raise ValueError(f"bad rank {rank} of {world}")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def batch_sharded_gemm(A: torch.Tensor, B: torch.Tensor, rank: int, world: int,
                       C: Optional[torch.Tensor] = None, **kw) -> torch.Tensor:
    """Local part of a batch-sharded strided batched GEMM.

    A, B are either the full [batch, ...] tensors (the local slice is taken as
    a view) or already-local slices when `C` is given with the local shape."""
    b0, b1 = shard_range(A.size(0), rank, world)
    return ops.batched_gemm(A[b0:b1], B[b0:b1], None if C is None else C[b0:b1], **kw)


@dataclass
class ColumnShardedGemm:
    """Y = X @ W with W split by columns over `world` ranks.

    w_local: this rank's contiguous [K, N/G] column block (N divisible by G).
    gemm_fn / gather_fn default to the library's kernels; tests of the host
    logic on CPU ranks substitute plain torch equivalents.
    """

    w_local: torch.Tensor
    world: int
    group: Optional[dist.ProcessGroup] = None
    chunks: int = 4
    gemm_fn: Optional[Callable] = None
    gather_fn: Optional[Callable] = None

    def _gemm(self, X, W, out):
        return (self.gemm_fn or ops.gemm)(X, W, out)

    def _gather(self, blocks, out):
        return (self.gather_fn or ops.gather_column_blocks)(blocks, out)

    def local(self, X: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """This rank's [M, N/G] output block (no communication)."""
        return self._gemm(X, self.w_local, out)

    def forward(self, X: torch.Tensor, gather: bool = True, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        if not gather or self.world == 1:
            return self.local(X, out)
        M, nb = X.size(0), self.w_local.size(1)
        G = self.world
        if out is None:
            out = torch.empty((M, G * nb), dtype=X.dtype, device=X.device)
        chunks = max(1, min(self.chunks, M))
        local_blk = torch.empty((M, nb), dtype=X.dtype, device=X.device)
        pending = []
        # Each chunk's all-gather is queued as soon as its rows are computed;
        # NCCL runs it on its own stream while the next chunk's GEMM runs.
        for c in range(chunks):
            r0, r1 = shard_range(M, c, chunks)
            if r1 <= r0:
                continue
            self._gemm(X[r0:r1], self.w_local, local_blk[r0:r1])
            recv = torch.empty((G * (r1 - r0), nb), dtype=X.dtype, device=X.device)
            try:
                h = dist.all_gather_into_tensor(recv, local_blk[r0:r1], group=self.group, async_op=True)
            except Exception as e:  # the backend refused the collective (a peer is gone)
                raise self._failed(r0, r1, e) from e
            pending.append((r0, r1, recv.view(G, r1 - r0, nb), h))
        for r0, r1, recv, h in pending:
            try:
                h.wait()  # the current stream waits for this chunk's collective
            except Exception as e:  # timed out, peer connection closed, or communicator aborted
                raise self._failed(r0, r1, e) from e
            self._gather(recv, out[r0:r1])
        return out

    @staticmethod
    def _failed(r0: int, r1: int, e: Exception) -> CollectiveError:
        return CollectiveError(f"all-gather of output rows {r0}:{r1} did not complete: a rank died, left or did not "
                               f"join within the process group's timeout ({type(e).__name__}: {e})")


def split_columns(W: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Contiguous copy of this rank's column block of a row-major [K, N] W."""
    n0, n1 = shard_range(W.size(1), rank, world)
    return W[:, n0:n1].contiguous()
