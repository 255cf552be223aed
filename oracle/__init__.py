"""Oracle for the cuop_b200 hot path — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
arm may import this package; the product (cuop_b200) never does.

Two oracles:
  * liboracle.so (cpu_ref.c): CPU restatement of the reference's GEMM / GEMV /
    batched math and summation order, plus the seeded input generator shared
    by tests and the bench.  Pinned against the reference's own known-answer
    tests (tests/golden/*.json, read from the reference's GTest sources).
  * _ref/libcuop_ref.so: the reference's own fp32 operators
    (Gemm<float>, Gemv<float>, BatchMatMul<float>) compiled from its sources
    by oracle/Makefile; GPU only.  Used to pin the CPU restatement and the
    CUDA kernels at the fp32 benchmark sizes.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
_LIB = HERE / "liboracle.so"
_REF = HERE / "_ref" / "libcuop_ref.so"
_lib = None
_ref = None

F16, BF16 = 2, 3
_i64, _f32, _f64, _vp, _int, _u64 = C.c_int64, C.c_float, C.c_double, C.c_void_p, C.c_int, C.c_uint64


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not _LIB.exists():
            raise ImportError(f"{_LIB} missing: run `make -C oracle`")
        L = C.CDLL(str(_LIB))
        sig = {
            "oracle_fill_uniform_f32": [_vp, _i64, _u64, _f32, _f32],
            "oracle_fill_normal_f32": [_vp, _i64, _u64, _f64, _f64],
            "oracle_f32_to_lowp": [_int, _vp, _vp, _i64],
            "oracle_lowp_to_f32": [_int, _vp, _vp, _i64],
            "oracle_gemm_f32": [_int, _int, _i64, _i64, _i64, _f32, _vp, _i64, _vp, _i64, _f32, _vp, _i64, _int],
            "oracle_gemm_f64": [_int, _int, _i64, _i64, _i64, _f64, _vp, _i64, _vp, _i64, _f64, _vp, _i64, _int],
            "oracle_gemm_lowp": [_int, _int, _int, _i64, _i64, _i64, _f32, _vp, _i64, _vp, _i64, _f32, _vp, _i64,
                                 _int],
            "oracle_gemm_lowp_ex": [_int, _int, _int, _i64, _i64, _i64, _f32, _vp, _i64, _vp, _i64, _f32, _vp,
                                    _i64, _vp, _int, _int],
            "oracle_epilogue_f32": [_i64, _i64, _vp, _i64, _vp, _int],
            "oracle_epilogue_f64": [_i64, _i64, _vp, _i64, _vp, _int],
            "oracle_gemm_batched_lowp": [_int, _int, _int, _i64, _i64, _i64, _f32, _vp, _i64, _i64, _vp, _i64, _i64,
                                         _f32, _vp, _i64, _i64, _i64, _int],
            "oracle_gemm_batched_f32": [_int, _int, _i64, _i64, _i64, _f32, _vp, _i64, _i64, _vp, _i64, _i64, _f32,
                                        _vp, _i64, _i64, _i64, _int],
            "oracle_gemm_sample_f64": [_int, _int, _i64, _vp, _i64, _vp, _i64, _vp, _i64, _vp, _i64, _vp, _int],
            "oracle_gemv_f32": [_int, _i64, _i64, _f32, _vp, _i64, _vp, _f32, _vp, _int],
            "oracle_gemv_f64acc": [_int, _i64, _i64, _vp, _i64, _vp, _vp, _int],
            "oracle_max_threads": [],
        }
        for name, args in sig.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = _int if name == "oracle_max_threads" else None
        _lib = L
    return _lib


def _p(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"] or a.ndim <= 1
    return a.ctypes.data


def threads() -> int:
    """Host threads available to this process (its CPU affinity), not
    OMP_NUM_THREADS: launchers such as torch.distributed.run set that to 1
    per worker, and the CPU baselines are meant to use the whole host.  Every
    oracle call passes its thread count explicitly."""
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except (AttributeError, OSError):
        return max(1, int(lib().oracle_max_threads()))


# ------------------------------------------------------------ generators
def uniform(shape, seed: int, lo: float = -1.0, hi: float = 1.0) -> np.ndarray:
    out = np.empty(shape, dtype=np.float32)
    lib().oracle_fill_uniform_f32(_p(out), out.size, seed, lo, hi)
    return out


def normal(shape, seed: int, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    out = np.empty(shape, dtype=np.float32)
    lib().oracle_fill_normal_f32(_p(out), out.size, seed, mean, std)
    return out


def to_lowp(a: np.ndarray, dtype: int) -> np.ndarray:
    """fp32 -> fp16/bf16 bits (uint16), round to nearest even."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    out = np.empty(a.shape, dtype=np.uint16)
    lib().oracle_f32_to_lowp(dtype, _p(a), _p(out), a.size)
    return out


def from_lowp(h: np.ndarray, dtype: int) -> np.ndarray:
    h = np.ascontiguousarray(h, dtype=np.uint16)
    out = np.empty(h.shape, dtype=np.float32)
    lib().oracle_lowp_to_f32(dtype, _p(h), _p(out), h.size)
    return out


# ------------------------------------------------------------ GEMM / GEMV
def _epi(bias, relu):
    return (1 if bias is not None else 0) | (2 if relu else 0)


def gemm_f32(A, B, C=None, transA=False, transB=False, alpha=1.0, beta=0.0, nthreads=None, bias=None, relu=False):
    """bias / relu: the fused epilogue of cuopx_gemm_ex (bias add, then ReLU)."""
    A = np.ascontiguousarray(A, np.float32)
    B = np.ascontiguousarray(B, np.float32)
    M, K = (A.shape[1], A.shape[0]) if transA else A.shape
    N = B.shape[0] if transB else B.shape[1]
    C = np.zeros((M, N), np.float32) if C is None else np.array(C, np.float32, copy=True)
    lib().oracle_gemm_f32(int(transA), int(transB), M, N, K, alpha, _p(A), A.shape[1], _p(B), B.shape[1], beta,
                          _p(C), N, nthreads or threads())
    if bias is not None or relu:
        bias = None if bias is None else np.ascontiguousarray(bias, np.float32)
        lib().oracle_epilogue_f32(M, N, _p(C), N, None if bias is None else _p(bias), _epi(bias, relu))
    return C


def gemm_f64(A, B, C=None, transA=False, transB=False, alpha=1.0, beta=0.0, nthreads=None, bias=None, relu=False):
    A = np.ascontiguousarray(A, np.float64)
    B = np.ascontiguousarray(B, np.float64)
    M, K = (A.shape[1], A.shape[0]) if transA else A.shape
    N = B.shape[0] if transB else B.shape[1]
    C = np.zeros((M, N), np.float64) if C is None else np.array(C, np.float64, copy=True)
    lib().oracle_gemm_f64(int(transA), int(transB), M, N, K, alpha, _p(A), A.shape[1], _p(B), B.shape[1], beta,
                          _p(C), N, nthreads or threads())
    if bias is not None or relu:
        bias = None if bias is None else np.ascontiguousarray(bias, np.float64)
        lib().oracle_epilogue_f64(M, N, _p(C), N, None if bias is None else _p(bias), _epi(bias, relu))
    return C


def gemm_lowp(dtype, A, B, C=None, transA=False, transB=False, alpha=1.0, beta=0.0, nthreads=None, bias=None,
              relu=False):
    """A, B, C (and bias) as uint16 bit patterns of fp16 (dtype=2) / bf16 (dtype=3)."""
    A = np.ascontiguousarray(A, np.uint16)
    B = np.ascontiguousarray(B, np.uint16)
    M, K = (A.shape[1], A.shape[0]) if transA else A.shape
    N = B.shape[0] if transB else B.shape[1]
    C = np.zeros((M, N), np.uint16) if C is None else np.array(C, np.uint16, copy=True)
    bias = None if bias is None else np.ascontiguousarray(bias, np.uint16)
    lib().oracle_gemm_lowp_ex(dtype, int(transA), int(transB), M, N, K, alpha, _p(A), A.shape[1], _p(B),
                              B.shape[1], beta, _p(C), N, None if bias is None else _p(bias), _epi(bias, relu),
                              nthreads or threads())
    return C


def gemm_batched_lowp(dtype, A, B, C=None, alpha=1.0, beta=0.0, nthreads=None):
    A = np.ascontiguousarray(A, np.uint16)
    B = np.ascontiguousarray(B, np.uint16)
    bt, M, K = A.shape
    N = B.shape[2]
    C = np.zeros((bt, M, N), np.uint16) if C is None else np.array(C, np.uint16, copy=True)
    lib().oracle_gemm_batched_lowp(dtype, 0, 0, M, N, K, alpha, _p(A), K, M * K, _p(B), N, K * N, beta, _p(C), N,
                                   M * N, bt, nthreads or threads())
    return C


def gemm_batched_f32(A, B, C=None, alpha=1.0, beta=0.0, nthreads=None):
    A = np.ascontiguousarray(A, np.float32)
    B = np.ascontiguousarray(B, np.float32)
    bt, M, K = A.shape
    N = B.shape[2]
    C = np.zeros((bt, M, N), np.float32) if C is None else np.array(C, np.float32, copy=True)
    lib().oracle_gemm_batched_f32(0, 0, M, N, K, alpha, _p(A), K, M * K, _p(B), N, K * N, beta, _p(C), N, M * N, bt,
                                  nthreads or threads())
    return C


def gemm_sample_f64(A, B, rows, cols, transA=False, transB=False, nthreads=None):
    """fp64-accumulated op(A) op(B) at rows x cols (A, B fp32 arrays)."""
    A = np.ascontiguousarray(A, np.float32)
    B = np.ascontiguousarray(B, np.float32)
    K = A.shape[0] if transA else A.shape[1]
    rows = np.ascontiguousarray(rows, np.int64)
    cols = np.ascontiguousarray(cols, np.int64)
    out = np.empty((rows.size, cols.size), np.float64)
    lib().oracle_gemm_sample_f64(int(transA), int(transB), K, _p(A), A.shape[1], _p(B), B.shape[1], _p(rows),
                                 rows.size, _p(cols), cols.size, _p(out), nthreads or threads())
    return out


def gemm_rows_cols_f64(A, B, rows, cols, block: int = 2048):
    """fp64 A @ B on complete rows and complete columns, for full-size error
    norms: returns (R, Q) with R = (A @ B)[rows, :] and Q = (A @ B)[:, cols].

    A [M, K] and B [K, N] are fp32 arrays (16-bit inputs already widened,
    exactly).  Every fp32 x fp32 product is exact in fp64, so this is the
    same fp64 reference value as gemm_sample_f64 up to fp64 summation order
    (~1e-16 relative); it runs as blocked fp64 matrix products, because a
    per-element loop over complete 8192-long rows and columns is far too
    slow on strided B.  Blocks of `block` columns (rows) bound the fp64
    copies to K x block."""
    A = np.asarray(A, np.float32)
    B = np.asarray(B, np.float32)
    M, K = A.shape
    N = B.shape[1]
    rows = np.asarray(rows, np.int64)
    cols = np.asarray(cols, np.int64)
    Ar = A[rows].astype(np.float64)
    R = np.empty((rows.size, N), np.float64)
    for j0 in range(0, N, block):
        j1 = min(N, j0 + block)
        R[:, j0:j1] = Ar @ B[:, j0:j1].astype(np.float64)
    Bc = B[:, cols].astype(np.float64)
    Q = np.empty((M, cols.size), np.float64)
    for i0 in range(0, M, block):
        i1 = min(M, i0 + block)
        Q[i0:i1] = A[i0:i1].astype(np.float64) @ Bc
    return R, Q


def gemv_f32(A, x, y=None, trans=False, alpha=1.0, beta=0.0, nthreads=None):
    A = np.ascontiguousarray(A, np.float32)
    x = np.ascontiguousarray(x, np.float32)
    N, M = A.shape if trans else (A.shape[1], A.shape[0])
    y = np.zeros(M, np.float32) if y is None else np.array(y, np.float32, copy=True)
    lib().oracle_gemv_f32(int(trans), M, N, alpha, _p(A), A.shape[1], _p(x), beta, _p(y), nthreads or threads())
    return y


def gemv_f64acc(A, x, trans=False, nthreads=None):
    A = np.ascontiguousarray(A, np.float32)
    x = np.ascontiguousarray(x, np.float32)
    N, M = A.shape if trans else (A.shape[1], A.shape[0])
    out = np.empty(M, np.float64)
    lib().oracle_gemv_f64acc(int(trans), M, N, _p(A), A.shape[1], _p(x), _p(out), nthreads or threads())
    return out


# ------------------------------------------------------------ tolerances
def rel_frobenius(C, R) -> float:
    """||C - R||_F / ||R||_F (fp32 path bound: 1e-5 * sqrt(K))."""
    C = np.asarray(C, np.float64)
    R = np.asarray(R, np.float64)
    den = np.linalg.norm(R)
    return float(np.linalg.norm(C - R) / (den if den > 0 else 1.0))


def max_relative(C, R) -> float:
    """max|C - R| / max|R| (fp16/bf16 path bound: 1e-2)."""
    C = np.asarray(C, np.float64)
    R = np.asarray(R, np.float64)
    den = np.max(np.abs(R)) if R.size else 1.0
    return float(np.max(np.abs(C - R)) / (den if den > 0 else 1.0)) if R.size else 0.0


# ------------------------------------------------------------ reference GPU oracle
def ref_available() -> bool:
    return _REF.exists()


def ref_lib() -> C.CDLL:
    """The reference's own fp32 operators (GPU); device pointers in, sync on return."""
    global _ref
    if _ref is None:
        L = C.CDLL(str(_REF))
        L.ref_gemm_f32.argtypes = [_int, _int, _int, _int, _int, _f32, _vp, _vp, _f32, _vp]
        L.ref_gemv_f32.argtypes = [_int, _int, _int, _f32, _vp, _vp, _f32, _vp]
        L.ref_batchmatmul_f32.argtypes = [_int, _int, _int, _int, _vp, _vp, _vp]
        L.ref_matmul_relu_f32.argtypes = [_int, _int, _int, _int, _int, _vp, _vp, _vp, _vp]
        for f in (L.ref_gemm_f32, L.ref_gemv_f32, L.ref_batchmatmul_f32, L.ref_matmul_relu_f32):
            f.restype = _int
        _ref = L
    return _ref
