"""Torch-tensor front end over the C ABI (include/cuopx.h).

Tensors only carry device memory and streams here: every call passes raw
device pointers to libcuopx.so, which launches the sm_100a kernels.  Shapes
and argument meaning follow cuOP's operators:

  gemm(A, B)        C = alpha * op(A) op(B) + beta * C   (Gemm<T>::Forward,
                    src/cuda_op/detail/cuBlas/gemm.cu:417-511)
  gemv(A, x)        y = alpha * op(A) x + beta * y        (Gemv<T>::Forward,
                    src/cuda_op/detail/cuBlas/gemv.cu:209-256)
  batched_gemm(A,B) C_b = alpha * A_b B_b + beta * C_b    (BatchMatMul<T>::Forward,
                    src/cuda_op/detail/cuDNN/batchmatmul.cu:52-94)
"""
from __future__ import annotations

import ctypes as C
import threading
from collections import OrderedDict
from typing import Optional

import torch

from . import _native as N

_DT = {torch.float32: N.F32, torch.float64: N.F64, torch.float16: N.F16, torch.bfloat16: N.BF16}

_ws_cache: dict = {}


def _dtype_code(t: torch.Tensor) -> int:
    try:
        return _DT[t.dtype]
    except KeyError:
        raise N.CuopError(N.UNSUPPORTED_TYPE, f"dtype {t.dtype}") from None


def _require_cuda(*ts: torch.Tensor) -> None:
    """Every tensor on one CUDA device (the kernels dereference all pointers there)."""
    dev = None
    for t in ts:
        if not t.is_cuda:
            raise N.CuopError(N.INVALID_ARGUMENT, "tensor is not on a CUDA device (no CPU path exists)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise N.CuopError(N.INVALID_ARGUMENT, f"tensors on {dev} and {t.device}")


def _row_ld(t: torch.Tensor) -> int:
    """Leading dimension of a row-major 2-D view (unit column stride)."""
    if t.dim() != 2 or (t.stride(1) != 1 and t.size(1) > 1):
        raise N.CuopError(N.INVALID_ARGUMENT, "expected a row-major 2-D tensor with unit column stride")
    return max(t.stride(0), t.size(1), 1)


def _stream(stream) -> int:
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, torch.cuda.Stream):
        return stream.cuda_stream
    return int(stream)


def workspace(nbytes: int, device: torch.device, tag: str = "ws") -> tuple[int, int]:
    """Per-device scratch (zeroed once at allocation); returns (ptr, bytes)."""
    if nbytes == 0:
        return 0, 0
    key = (tag, device.index if device.index is not None else torch.cuda.current_device())
    buf = _ws_cache.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _ws_cache[key] = buf
    return buf.data_ptr(), buf.numel()


def gemm(A: torch.Tensor, B: torch.Tensor, C: Optional[torch.Tensor] = None, *, transA: bool = False,
         transB: bool = False, alpha: float = 1.0, beta: float = 0.0, bias: Optional[torch.Tensor] = None,
         relu: bool = False, stream=None) -> torch.Tensor:
    """C = act(alpha * op(A) op(B) + beta * C + bias) for row-major 2-D tensors;
    bias ([N], same dtype) and relu select the fused epilogue (cuopx_gemm_ex)."""
    _require_cuda(A, B)
    M = A.size(1) if transA else A.size(0)
    K = A.size(0) if transA else A.size(1)
    Kb = B.size(1) if transB else B.size(0)
    Nn = B.size(0) if transB else B.size(1)
    if Kb != K:
        raise N.CuopError(N.SHAPE_MISMATCH, f"gemm: op(A) is {M}x{K}, op(B) is {Kb}x{Nn}")
    if A.dtype != B.dtype:
        raise N.CuopError(N.UNSUPPORTED_TYPE, "gemm: A and B must share a dtype")
    if C is None:
        C = torch.empty((M, Nn), dtype=A.dtype, device=A.device)
        beta = 0.0
    _require_cuda(A, B, C)
    if tuple(C.shape) != (M, Nn) or C.dtype != A.dtype:
        raise N.CuopError(N.SHAPE_MISMATCH, f"gemm: C must be {M}x{Nn} {A.dtype}")
    if bias is None and not relu:
        rc = N.lib().cuopx_gemm(_dtype_code(A), int(transA), int(transB), M, Nn, K, float(alpha), A.data_ptr(),
                                _row_ld(A), B.data_ptr(), _row_ld(B), float(beta), C.data_ptr(), _row_ld(C),
                                _stream(stream))
        N.check(rc, "cuopx_gemm")
        return C
    epi = N.EPI_RELU if relu else N.EPI_NONE
    bptr = 0
    if bias is not None:
        _require_cuda(A, bias)
        if bias.dtype != A.dtype or bias.numel() != Nn or not bias.is_contiguous():
            raise N.CuopError(N.SHAPE_MISMATCH, f"gemm: bias must be a contiguous [{Nn}] {A.dtype} vector")
        epi |= N.EPI_BIAS
        bptr = bias.data_ptr()
    rc = N.lib().cuopx_gemm_ex(_dtype_code(A), int(transA), int(transB), M, Nn, K, float(alpha), A.data_ptr(),
                               _row_ld(A), B.data_ptr(), _row_ld(B), float(beta), C.data_ptr(), _row_ld(C), bptr,
                               epi, _stream(stream))
    N.check(rc, "cuopx_gemm_ex")
    return C


def batched_gemm(A: torch.Tensor, B: torch.Tensor, C: Optional[torch.Tensor] = None, *, transA: bool = False,
                 transB: bool = False, alpha: float = 1.0, beta: float = 0.0, stream=None) -> torch.Tensor:
    """Strided batched GEMM over contiguous [batch, rows, cols] tensors."""
    _require_cuda(A, B)
    if A.dim() != 3 or B.dim() != 3:
        raise N.CuopError(N.SHAPE_MISMATCH, "batched_gemm expects 3-D tensors")
    A = A if A.is_contiguous() else A.contiguous()
    B = B if B.is_contiguous() else B.contiguous()
    batch = A.size(0)
    M = A.size(2) if transA else A.size(1)
    K = A.size(1) if transA else A.size(2)
    Kb = B.size(2) if transB else B.size(1)
    Nn = B.size(1) if transB else B.size(2)
    if Kb != K or B.size(0) != batch:
        raise N.CuopError(N.SHAPE_MISMATCH, "batched_gemm: shape mismatch")
    if C is None:
        C = torch.empty((batch, M, Nn), dtype=A.dtype, device=A.device)
        beta = 0.0
    _require_cuda(A, B, C)
    if tuple(C.shape) != (batch, M, Nn) or not C.is_contiguous():
        raise N.CuopError(N.SHAPE_MISMATCH, "batched_gemm: bad C")
    rc = N.lib().cuopx_gemm_strided_batched(
        _dtype_code(A), int(transA), int(transB), M, Nn, K, float(alpha), A.data_ptr(), A.size(2),
        A.size(1) * A.size(2), B.data_ptr(), B.size(2), B.size(1) * B.size(2), float(beta), C.data_ptr(), Nn,
        M * Nn, batch, _stream(stream))
    N.check(rc, "cuopx_gemm_strided_batched")
    return C


class _HostStreamer:
    """Device staging for batched_gemm_host on one device: `slots` chunk
    buffers for A, B and C, a host-to-device and a device-to-host copy
    stream, and one event per slot and stage.  Kept between calls (a call
    after the first allocates nothing); `lock` serialises calls that share
    it (several host threads with the same shape)."""

    def __init__(self, device: torch.device, dtype: torch.dtype, chunk: int, shapes, slots: int):
        (m, k), (k2, n) = shapes
        self.key = (device, dtype, chunk, m, k, n, slots)
        self.slots = slots
        self.lock = threading.Lock()
        self.dA = [torch.empty((chunk, m, k), dtype=dtype, device=device) for _ in range(slots)]
        self.dB = [torch.empty((chunk, k2, n), dtype=dtype, device=device) for _ in range(slots)]
        self.dC = [torch.empty((chunk, m, n), dtype=dtype, device=device) for _ in range(slots)]
        self.h2d = torch.cuda.Stream(device)
        self.d2h = torch.cuda.Stream(device)
        self.loaded = [torch.cuda.Event() for _ in range(slots)]
        self.computed = [torch.cuda.Event() for _ in range(slots)]
        self.stored = [torch.cuda.Event() for _ in range(slots)]


# Staging sets by (device, dtype, chunk, shape, slots), least recently used
# first; at most _MAX_STREAMERS are kept.
_streamers: "OrderedDict" = OrderedDict()
_streamers_lock = threading.Lock()
_MAX_STREAMERS = 4


def batched_gemm_host(A: torch.Tensor, B: torch.Tensor, C: torch.Tensor, *, alpha: float = 1.0, beta: float = 0.0,
                      device: Optional[torch.device] = None, chunk: Optional[int] = None,
                      slots: int = 3) -> torch.Tensor:
    """C_b = alpha * A_b B_b + beta * C_b for PINNED HOST tensors [batch, ...]:
    the batch streams through `device` (default: the current one) in chunks.
    The host-to-device copy of chunk i+1, the batched GEMM of chunk i
    (cuopx_gemm_strided_batched on the current stream) and the device-to-host
    copy of chunk i-1 overlap, each copy direction on its own stream, so both
    PCIe directions and the GPU are busy at once.  Returns after C holds the
    result (the host has waited for the last copy).  The reference's
    BatchMatMul<T>::Forward (src/cuda_op/detail/cuDNN/batchmatmul.cu:52-94)
    takes device tensors; this is the same product for data that starts and
    ends in host memory."""
    for t, nm in ((A, "A"), (B, "B"), (C, "C")):
        if t.is_cuda or not t.is_pinned() or not t.is_contiguous() or t.dim() != 3:
            raise N.CuopError(N.INVALID_ARGUMENT, f"batched_gemm_host: {nm} must be a contiguous 3-D pinned host tensor")
    if not (A.dtype == B.dtype == C.dtype):
        raise N.CuopError(N.UNSUPPORTED_TYPE, "batched_gemm_host: A, B and C must share a dtype")
    batch, M, K = A.shape
    if B.size(0) != batch or B.size(1) != K or tuple(C.shape) != (batch, M, B.size(2)):
        raise N.CuopError(N.SHAPE_MISMATCH, "batched_gemm_host: shape mismatch")
    if batch == 0:
        return C
    dev = device or torch.device("cuda", torch.cuda.current_device())
    per_batch = (M * K + K * B.size(2) + M * B.size(2)) * A.element_size()
    if chunk is None:  # about 8 chunks, each moving at least 8 MiB (measured best on B200 over PCIe 5)
        chunk = max(1, min(batch, max((8 << 20) // per_batch, -(-batch // 8))))
    # Chunk boundaries: the first and the last chunk are a quarter size, so
    # that the copy-in before the first GEMM and the copy-out after the last
    # one, which nothing overlaps, are short.  (Measured on a C4 step over
    # PCIe 5: the copy-in direction is busy throughout at ~42 GB/s while the
    # copy-out runs beside it; quarter-size edges gain ~1 % over half-size.)
    bounds = []
    b0 = 0
    edge = max(1, chunk // 4)
    while b0 < batch:
        rest = batch - b0
        n = edge if b0 == 0 else chunk
        if b0 > 0 and rest <= chunk + edge:  # tail: split what is left into two, the last one edge-sized
            n = rest - edge if rest > edge else rest
        n = min(n, rest)
        bounds.append((b0, b0 + n))
        b0 += n
    key = (dev, A.dtype, chunk, M, K, B.size(2), slots)
    with _streamers_lock:
        st = _streamers.get(key)
        if st is None:
            st = _HostStreamer(dev, A.dtype, chunk, ((M, K), (K, B.size(2))), slots)
            _streamers[key] = st
            while len(_streamers) > _MAX_STREAMERS:  # drop the least recently used (idle: calls end synchronised)
                old_key, old_st = next(iter(_streamers.items()))
                if old_st.lock.locked():
                    break
                del _streamers[old_key]
        _streamers.move_to_end(key)
    with st.lock:
        return _stream_batches(st, A, B, C, alpha, beta, bounds, dev)


def _stream_batches(st: "_HostStreamer", A, B, C, alpha, beta, bounds, dev):
    slots = st.slots
    comp = torch.cuda.current_stream(dev)
    last = None
    with torch.cuda.device(dev):
        for c, (b0, b1) in enumerate(bounds):
            n, s = b1 - b0, c % slots
            with torch.cuda.stream(st.h2d):
                if c >= slots:
                    st.h2d.wait_event(st.computed[s])  # the GEMM of chunk c - slots has read this slot
                st.dA[s][:n].copy_(A[b0:b1], non_blocking=True)
                st.dB[s][:n].copy_(B[b0:b1], non_blocking=True)
                if beta != 0.0:
                    if c >= slots:
                        st.h2d.wait_event(st.stored[s])  # and its C has left the slot
                    st.dC[s][:n].copy_(C[b0:b1], non_blocking=True)
                st.loaded[s].record(st.h2d)
            comp.wait_event(st.loaded[s])
            if c >= slots:
                comp.wait_event(st.stored[s])
            batched_gemm(st.dA[s][:n], st.dB[s][:n], st.dC[s][:n], alpha=alpha, beta=beta, stream=comp)
            st.computed[s].record(comp)
            with torch.cuda.stream(st.d2h):
                st.d2h.wait_event(st.computed[s])
                C[b0:b1].copy_(st.dC[s][:n], non_blocking=True)
                st.stored[s].record(st.d2h)
            last = st.stored[s]
    last.synchronize()
    return C


def gemv(A: torch.Tensor, x: torch.Tensor, y: Optional[torch.Tensor] = None, *, trans: bool = False,
         alpha: float = 1.0, beta: float = 0.0, stream=None) -> torch.Tensor:
    """y = alpha * op(A) x + beta * y.

    trans=False: A is M x N, x has N entries, y has M.
    trans=True:  A is N x M (the reference reads A[col*m+row]); y = A^T x has M.
    y may also be a pinned host tensor: the kernel then writes the result
    straight into host memory (zero-copy), with no device-to-host copy.
    """
    _require_cuda(A, x)
    if x.dtype != A.dtype or not x.is_contiguous():
        raise N.CuopError(N.INVALID_ARGUMENT, f"gemv: x must be a contiguous {A.dtype} vector")
    if trans:
        Nn, M = A.size(0), A.size(1)
    else:
        M, Nn = A.size(0), A.size(1)
    if x.numel() != Nn:
        raise N.CuopError(N.SHAPE_MISMATCH, f"gemv: x has {x.numel()} entries, expected {Nn}")
    if y is None:
        y = torch.empty(M, dtype=A.dtype, device=A.device)
        beta = 0.0
    if y.numel() != M:
        raise N.CuopError(N.SHAPE_MISMATCH, f"gemv: y has {y.numel()} entries, expected {M}")
    if y.dtype != A.dtype or not y.is_contiguous():
        raise N.CuopError(N.INVALID_ARGUMENT, f"gemv: y must be a contiguous {A.dtype} vector")
    if y.is_cuda:
        _require_cuda(A, y)
    elif not y.is_pinned():
        raise N.CuopError(N.INVALID_ARGUMENT, "gemv: y must be on A's device or in pinned host memory")
    dt = _dtype_code(A)
    need = N.lib().cuopx_gemv_workspace_size(dt, int(trans), M, Nn)
    ws, wsb = workspace(need, A.device)
    rc = N.lib().cuopx_gemv(dt, int(trans), M, Nn, float(alpha), A.data_ptr(), _row_ld(A), x.data_ptr(),
                            float(beta), y.data_ptr(), ws, wsb, _stream(stream))
    N.check(rc, "cuopx_gemv")
    return y


def gather_column_blocks(blocks: torch.Tensor, out: torch.Tensor, stream=None) -> torch.Tensor:
    """blocks: [G, M, Nb] contiguous -> out: [M, G*Nb] row-major."""
    _require_cuda(blocks, out)
    G, M, Nb = blocks.shape
    if not blocks.is_contiguous() or out.size(0) != M or out.size(1) != G * Nb or out.dtype != blocks.dtype:
        raise N.CuopError(N.SHAPE_MISMATCH, "gather_column_blocks: out must be [M, G*Nb] of the blocks' dtype")
    rc = N.lib().cuopx_gather_column_blocks(_dtype_code(blocks), G, M, Nb, blocks.data_ptr(), out.data_ptr(),
                                            _row_ld(out), _stream(stream))
    N.check(rc, "cuopx_gather_column_blocks")
    return out


# ----------------------------------------------------------------- level 1
def _vws(x: torch.Tensor) -> tuple[int, int]:
    return workspace(N.lib().cuopx_vector_workspace_size(x.numel()), x.device, tag="vec")


def _f32(*ts):
    for t in ts:
        if t.dtype != torch.float32:
            raise N.CuopError(N.UNSUPPORTED_TYPE, "vector ops are fp32")
    _require_cuda(*ts)


def dot(x, y, n=None, incx=1, incy=1, stream=None) -> torch.Tensor:
    _f32(x, y)
    n = x.numel() if n is None else n
    out = torch.empty(1, dtype=torch.float32, device=x.device)
    ws, wsb = _vws(x)
    N.check(N.lib().cuopx_dot(n, x.data_ptr(), incx, y.data_ptr(), incy, out.data_ptr(), ws, wsb, _stream(stream)),
            "cuopx_dot")
    return out


def nrm2(x, n=None, incx=1, stream=None) -> torch.Tensor:
    _f32(x)
    n = x.numel() if n is None else n
    out = torch.empty(1, dtype=torch.float32, device=x.device)
    ws, wsb = _vws(x)
    N.check(N.lib().cuopx_nrm2(n, x.data_ptr(), incx, out.data_ptr(), ws, wsb, _stream(stream)), "cuopx_nrm2")
    return out


def asum(x, n=None, incx=1, stream=None) -> torch.Tensor:
    _f32(x)
    n = x.numel() if n is None else n
    out = torch.empty(1, dtype=torch.float32, device=x.device)
    ws, wsb = _vws(x)
    N.check(N.lib().cuopx_asum(n, x.data_ptr(), incx, out.data_ptr(), ws, wsb, _stream(stream)), "cuopx_asum")
    return out


def iamax(x, n=None, incx=1, stream=None) -> torch.Tensor:
    _f32(x)
    n = x.numel() if n is None else n
    out = torch.empty(1, dtype=torch.int64, device=x.device)
    ws, wsb = _vws(x)
    N.check(N.lib().cuopx_iamax(n, x.data_ptr(), incx, out.data_ptr(), ws, wsb, _stream(stream)), "cuopx_iamax")
    return out


def iamin(x, n=None, incx=1, stream=None) -> torch.Tensor:
    _f32(x)
    n = x.numel() if n is None else n
    out = torch.empty(1, dtype=torch.int64, device=x.device)
    ws, wsb = _vws(x)
    N.check(N.lib().cuopx_iamin(n, x.data_ptr(), incx, out.data_ptr(), ws, wsb, _stream(stream)), "cuopx_iamin")
    return out


def axpy(alpha, x, y, n=None, incx=1, incy=1, stream=None):
    _f32(x, y)
    n = x.numel() if n is None else n
    N.check(N.lib().cuopx_axpy(n, float(alpha), x.data_ptr(), incx, y.data_ptr(), incy, _stream(stream)), "cuopx_axpy")
    return y


def scal(alpha, x, n=None, incx=1, stream=None):
    _f32(x)
    n = x.numel() if n is None else n
    N.check(N.lib().cuopx_scal(n, float(alpha), x.data_ptr(), incx, _stream(stream)), "cuopx_scal")
    return x


def copy(x, y, n=None, incx=1, incy=1, stream=None):
    """y = x.  One side may be a pinned host tensor: the kernel then reads or
    writes host memory directly (staging with no copy-engine transfer)."""
    for t in (x, y):
        if t.dtype != torch.float32:
            raise N.CuopError(N.UNSUPPORTED_TYPE, "vector ops are fp32")
    on_dev = [t for t in (x, y) if t.is_cuda]
    if not on_dev or any(not t.is_cuda and not t.is_pinned() for t in (x, y)):
        raise N.CuopError(N.INVALID_ARGUMENT, "copy: one side on a CUDA device, the other there or in pinned host memory")
    _require_cuda(*on_dev)
    n = x.numel() if n is None else n
    N.check(N.lib().cuopx_copy(n, x.data_ptr(), incx, y.data_ptr(), incy, _stream(stream)), "cuopx_copy")
    return y


def swap(x, y, n=None, incx=1, incy=1, stream=None):
    _f32(x, y)
    n = x.numel() if n is None else n
    N.check(N.lib().cuopx_swap(n, x.data_ptr(), incx, y.data_ptr(), incy, _stream(stream)), "cuopx_swap")
    return x, y


def rot(x, y, c, s, n=None, incx=1, incy=1, stream=None):
    _f32(x, y)
    n = x.numel() if n is None else n
    N.check(N.lib().cuopx_rot(n, x.data_ptr(), incx, y.data_ptr(), incy, float(c), float(s), _stream(stream)),
            "cuopx_rot")
    return x, y


# ----------------------------------------------------------------- diagnostics
def last_kernel() -> str:
    return N.lib().cuopx_last_kernel().decode()


def launch_count() -> int:
    return int(N.lib().cuopx_launch_count())


def device_error() -> int:
    v = C.c_int(0)
    N.check(N.lib().cuopx_get_device_error(C.byref(v)), "cuopx_get_device_error")
    return v.value


def clear_device_error() -> None:
    N.check(N.lib().cuopx_clear_device_error(), "cuopx_clear_device_error")
