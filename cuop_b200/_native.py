"""ctypes binding of libcuopx.so (the C ABI declared in include/cuopx.h).

The library must exist (built by cuop_b200.build / __graft_entry__.build());
there is no fallback of any kind: a missing or unloadable library raises.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

_LIB_PATH = Path(__file__).resolve().parent / "libcuopx.so"
_lib = None

# Status codes (numerically identical to cuOP's StatusCode).
SUCCESS = 0
NOT_IMPLEMENTED = 1001
TIMEOUT = 1003
RESOURCE_UNAVAILABLE = 1005
CUDA_ERROR = 2000
OUT_OF_MEMORY = 3001
INVALID_ARGUMENT = 4001
EXECUTION_TIMEOUT = 6002
KERNEL_NOT_FOUND = 6005
NOT_COMPILED = 7003
SHAPE_MISMATCH = 10002
UNSUPPORTED_TYPE = 11001

STATUS_NAMES = {
    0: "SUCCESS", 1001: "NOT_IMPLEMENTED", 1003: "TIMEOUT", 1005: "RESOURCE_UNAVAILABLE", 2000: "CUDA_ERROR", 3001: "OUT_OF_MEMORY",
    4001: "INVALID_ARGUMENT", 6002: "EXECUTION_TIMEOUT", 6005: "KERNEL_NOT_FOUND", 7003: "NOT_COMPILED",
    10002: "SHAPE_MISMATCH", 11001: "UNSUPPORTED_TYPE",
}

F32, F64, F16, BF16 = 0, 1, 2, 3
FP32_AUTO, FP32_FFMA, FP32_TF32X3 = 0, 1, 2
EPI_NONE, EPI_BIAS, EPI_RELU = 0, 1, 2
PEER_HANDLE_BYTES = 64
PEER_SIGNAL_BYTES = 512
DEVERR_PEER_TIMEOUT = 8

_i64, _dbl, _vp, _sz, _int = C.c_int64, C.c_double, C.c_void_p, C.c_size_t, C.c_int
_fp = C.c_void_p  # float* as raw address

# (name, restype, argtypes) for every symbol in include/cuopx.h
SIGNATURES = [
    ("cuopx_version", _int, []),
    ("cuopx_set_fp32_gemm_mode", _int, [_int]),
    ("cuopx_get_fp32_gemm_mode", _int, []),
    ("cuopx_last_kernel", C.c_char_p, []),
    ("cuopx_last_cuda_error", C.c_char_p, []),
    ("cuopx_launch_count", _i64, []),
    ("cuopx_get_device_error", _int, [C.POINTER(_int)]),
    ("cuopx_clear_device_error", _int, []),
    ("cuopx_tuning_load", _int, [C.c_char_p]),
    ("cuopx_tuning_load_file", _int, [C.c_char_p]),
    ("cuopx_tuning_clear", _int, []),
    ("cuopx_tuning_rows", _int, []),
    ("cuopx_set_gemm_variant", _int, [C.c_char_p]),
    ("cuopx_set_gemm_variant_thread", _int, [C.c_char_p]),
    ("cuopx_gemm_variant_name", C.c_char_p, [_int]),
    ("cuopx_gemm", _int, [_int, _int, _int, _i64, _i64, _i64, _dbl, _vp, _i64, _vp, _i64, _dbl, _vp, _i64, _vp]),
    ("cuopx_gemm_ex", _int,
     [_int, _int, _int, _i64, _i64, _i64, _dbl, _vp, _i64, _vp, _i64, _dbl, _vp, _i64, _vp, _int, _vp]),
    ("cuopx_gemm_strided_batched", _int,
     [_int, _int, _int, _i64, _i64, _i64, _dbl, _vp, _i64, _i64, _vp, _i64, _i64, _dbl, _vp, _i64, _i64, _i64, _vp]),
    ("cuopx_gemv_workspace_size", _sz, [_int, _int, _i64, _i64]),
    ("cuopx_gemv", _int, [_int, _int, _i64, _i64, _dbl, _vp, _i64, _vp, _dbl, _vp, _vp, _sz, _vp]),
    ("cuopx_gemv_noalloc", _int, [_int, _int, _i64, _i64, _dbl, _vp, _i64, _vp, _dbl, _vp, _vp]),
    ("cuopx_gather_column_blocks", _int, [_int, _i64, _i64, _i64, _vp, _vp, _i64, _vp]),
    ("cuopx_peer_alloc", _int, [_sz, C.POINTER(_vp), _vp]),
    ("cuopx_peer_open", _int, [_vp, C.POINTER(_vp)]),
    ("cuopx_peer_close", _int, [_vp]),
    ("cuopx_peer_free", _int, [_vp]),
    ("cuopx_peer_barrier", _int, [C.POINTER(_vp), _int, _int, _vp]),
    ("cuopx_gemm_allgather", _int,
     [_int, _int, _int, _i64, _i64, _i64, _dbl, _vp, _i64, _vp, _i64, C.POINTER(_vp), _int, _int, _i64, _vp]),
    ("cuopx_vector_workspace_size", _sz, [_i64]),
    ("cuopx_dot", _int, [_i64, _fp, _i64, _fp, _i64, _fp, _vp, _sz, _vp]),
    ("cuopx_axpy", _int, [_i64, C.c_float, _fp, _i64, _fp, _i64, _vp]),
    ("cuopx_scal", _int, [_i64, C.c_float, _fp, _i64, _vp]),
    ("cuopx_copy", _int, [_i64, _fp, _i64, _fp, _i64, _vp]),
    ("cuopx_swap", _int, [_i64, _fp, _i64, _fp, _i64, _vp]),
    ("cuopx_rot", _int, [_i64, _fp, _i64, _fp, _i64, C.c_float, C.c_float, _vp]),
    ("cuopx_nrm2", _int, [_i64, _fp, _i64, _fp, _vp, _sz, _vp]),
    ("cuopx_asum", _int, [_i64, _fp, _i64, _fp, _vp, _sz, _vp]),
    ("cuopx_iamax", _int, [_i64, _fp, _i64, _vp, _vp, _sz, _vp]),
    ("cuopx_iamin", _int, [_i64, _fp, _i64, _vp, _vp, _sz, _vp]),
]


class CuopError(RuntimeError):
    def __init__(self, code: int, what: str):
        super().__init__(f"{what}: {STATUS_NAMES.get(code, code)} ({code})")
        self.code = code


def lib_path() -> Path:
    return _LIB_PATH


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not _LIB_PATH.exists():
            raise ImportError(f"{_LIB_PATH} is missing: run `python -m cuop_b200.build` (no fallback path exists)")
        handle = C.CDLL(str(_LIB_PATH))
        for name, res, args in SIGNATURES:
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        # GEMM variant table from the offline sweep (cuop_b200/tuning.py).
        table = _LIB_PATH.parent / "tuning_b200.txt"
        if table.exists():
            check(handle.cuopx_tuning_load_file(str(table).encode()), f"cuopx_tuning_load_file({table})")
        _lib = handle
    return _lib


def check(code: int, what: str) -> None:
    if code != SUCCESS:
        if code == CUDA_ERROR:
            what = f"{what} [{lib().cuopx_last_cuda_error().decode()}]"
        raise CuopError(code, what)
