"""ctypes binding of libecq.so (the C ABI declared in include/ecq.h).

The shared library is built in-tree by ``ecq_b200.build`` and loaded from
``ecq_b200/_lib/libecq.so``. There is no fallback: if the library is missing
or does not export the expected symbols, loading fails with an error.
"""
from __future__ import annotations

import ctypes
from ctypes import POINTER, c_int32, c_int64, c_uint16, c_uint32, c_uint64, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libecq.so"

ECQ_OK = 0
ERRORS = {
    -1: "bad argument",
    -2: "unsupported or inconsistent shape",
    -3: "frequency table does not sum to 16384",
    -4: "a symbol that occurs has frequency 0",
    -5: "output buffer too small",
    -6: "CUDA error",
    -7: "internal error",
    -8: "configuration not supported by the compiled kernels",
    -9: "workspace missing or too small",
}
STATUS_CORRUPT = 1
STATUS_TIMEOUT = 2
STATUS_BADARG = 4
FLAG_CONSTANT = 1
TILE_ROWS = 8
NOALLOC_SCRATCH_BYTES = 4 << 20
TABLE_ENTRIES = 16384
TP_MAX_RANKS = 8
IPC_HANDLE_BYTES = 64

# every function include/*.h declares
EXPORTS = (
    "ecq_version",
    "ecq_table_from_counts",
    "ecq_build_decode_table",
    "ecq_encode_interleaved_host",
    "ecq_matrix_encoded_bound",
    "ecq_encode_matrix_host",
    "ecq_decode_interleaved",
    "ecq_matrix_decode",
    "ecq_matrix_decode_packed4",
    "ecq_matrix_dequantize",
    "ecq_gemv_workspace_bytes",
    "ecq_gemv",
    "ecq_gemv_fused",
    "ecq_gemv_noalloc",
    "ecq_plain4_gemv",
    "ecq_matmul_workspace_bytes",
    "ecq_matmul",
    "ecq_device_info",
    "ecq_comm_buffer_bytes",
    "ecq_comm_alloc",
    "ecq_comm_free",
    "ecq_ipc_get_handle",
    "ecq_ipc_open",
    "ecq_ipc_close",
    "ecq_gemv_tp",
    "ecq_tp_add_rmsnorm_f16",
    "ecq_tp_sum_f16",
    "ecq_add_rmsnorm_f16",
    "ecq_rope_kv_f16",
    "ecq_silu_mul_f16",
    "ecq_decode_attention_workspace_bytes",
    "ecq_decode_attention_splits",
    "ecq_decode_attention_f16",
)


class EcqError(RuntimeError):
    pass


class MatrixView(ctypes.Structure):
    """Mirror of ``ecq_matrix_view``."""

    _fields_ = [
        ("rows", c_uint32), ("cols", c_uint32),
        ("tile_rows", c_uint32), ("tile_cols", c_uint32),
        ("group_size", c_uint32), ("n_tiles", c_uint32),
        ("max_tile_bytes", c_uint32), ("flags", c_uint32),
        ("data", c_void_p), ("tile_offset", c_void_p),
        ("stream_len", c_void_p), ("dec_table", c_void_p),
    ]


EPI_ROPE_KV = 1
EPI_SILU_MUL = 2


class GemvEpilogue(ctypes.Structure):
    """Mirror of ``ecq_gemv_epilogue``."""

    _fields_ = [
        ("kind", c_int32), ("part_rows", c_uint32), ("head_dim", c_uint32), ("reserved", c_uint32),
        ("cache_head_stride", c_int64), ("cos_f16", c_void_p), ("sin_f16", c_void_p),
        ("k_cache_f16", c_void_p), ("v_cache_f16", c_void_p),
    ]


class TPComm(ctypes.Structure):
    """Mirror of ``ecq_tp_comm`` (include/ecq_comm.h)."""

    _fields_ = [
        ("world", c_uint32), ("rank", c_uint32), ("n_max", c_uint32), ("reserved", c_uint32),
        ("local", c_void_p), ("peers", c_void_p * TP_MAX_RANKS),
    ]


_lib = None


def _declare(L: ctypes.CDLL) -> None:
    P = c_void_p
    sig = {
        "ecq_version": (c_int32, []),
        "ecq_table_from_counts": (c_int32, [P, P, P]),
        "ecq_build_decode_table": (c_int32, [P, P, P]),
        "ecq_encode_interleaved_host": (c_int64, [P, c_int64, c_int32, P, P, c_int64, P, P]),
        "ecq_matrix_encoded_bound": (c_int64, [c_uint32, c_uint32, c_uint32, c_uint32]),
        "ecq_encode_matrix_host": (c_int32, [P, c_uint32, c_uint32, c_uint32, c_uint32, P, c_int32, P, c_int64, P, P, P]),
        "ecq_decode_interleaved": (c_int32, [P, P, c_uint32, c_uint64, c_uint32, P, c_uint32, P, P, P]),
        "ecq_matrix_decode": (c_int32, [POINTER(MatrixView), P, P, P]),
        "ecq_matrix_decode_packed4": (c_int32, [POINTER(MatrixView), P, P, P]),
        "ecq_matrix_dequantize": (c_int32, [POINTER(MatrixView), P, P, P, P]),
        "ecq_plain4_gemv": (c_int32, [P, P, P, P, c_uint32, c_uint32, c_uint32, c_uint32, P]),
        "ecq_gemv_workspace_bytes": (c_int64, [POINTER(MatrixView), c_uint32]),
        "ecq_gemv": (c_int32, [POINTER(MatrixView), P, P, P, c_uint32, P, c_int64, P, P]),
        "ecq_gemv_fused": (c_int32, [POINTER(MatrixView), P, P, P, POINTER(GemvEpilogue), P, c_int64, P, P]),
        "ecq_gemv_noalloc": (c_int32, [POINTER(MatrixView), P, P, P, c_uint32, P, P]),
        "ecq_matmul_workspace_bytes": (c_int64, [POINTER(MatrixView), c_uint32]),
        "ecq_matmul": (c_int32, [POINTER(MatrixView), P, P, P, c_uint32, P, c_int64, P, P]),
        "ecq_device_info": (c_int32, [P, P, P, POINTER(MatrixView)]),
        "ecq_comm_buffer_bytes": (c_int64, [c_uint32, c_uint32]),
        "ecq_comm_alloc": (c_int32, [c_int64, POINTER(c_void_p)]),
        "ecq_comm_free": (c_int32, [P]),
        "ecq_ipc_get_handle": (c_int32, [P, P]),
        "ecq_ipc_open": (c_int32, [P, POINTER(c_void_p)]),
        "ecq_ipc_close": (c_int32, [P]),
        "ecq_gemv_tp": (c_int32, [POINTER(MatrixView), P, P, POINTER(TPComm), P, c_int64, P, P]),
        "ecq_tp_add_rmsnorm_f16": (c_int32, [P, POINTER(TPComm), P, P, P, c_int32, ctypes.c_float, P, P]),
        "ecq_tp_sum_f16": (c_int32, [POINTER(TPComm), P, c_int32, P, P]),
        "ecq_add_rmsnorm_f16": (c_int32, [P, P, P, P, P, c_int32, c_int32, ctypes.c_float, P]),
        "ecq_rope_kv_f16": (c_int32, [P, P, P, P, P, P, P, c_int32, c_int32, c_int64, P]),
        "ecq_silu_mul_f16": (c_int32, [P, P, c_int32, c_int32, P]),
        "ecq_decode_attention_workspace_bytes": (c_int64, [c_int32, c_int32]),
        "ecq_decode_attention_splits": (c_int32, [c_int32, c_int32]),
        "ecq_decode_attention_f16": (c_int32, [P, P, P, P, c_int32, c_int32, c_int32, c_int64, c_int32, P, c_int64, P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args


def lib() -> ctypes.CDLL:
    """Load libecq.so (building it first if it is absent and nvcc exists)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            from . import build as _build

            _build.build()
        if not LIB_PATH.exists():
            raise EcqError(f"libecq.so not found at {LIB_PATH}; run python -m ecq_b200.build")
        L = ctypes.CDLL(str(LIB_PATH))
        missing = [s for s in EXPORTS if not hasattr(L, s)]
        if missing:
            raise EcqError(f"libecq.so lacks symbols: {missing}")
        _declare(L)
        _lib = L
    return _lib


def check(rc: int, what: str) -> int:
    if rc < 0:
        raise EcqError(f"{what}: {ERRORS.get(int(rc), 'error')} ({rc})")
    return rc


def ptr(a) -> int:
    """Raw address of a numpy array or torch tensor (None -> 0)."""
    if a is None:
        return 0
    if hasattr(a, "data_ptr"):
        return a.data_ptr()
    return a.ctypes.data


__all__ = ["lib", "check", "ptr", "MatrixView", "TPComm", "GemvEpilogue", "EcqError", "EXPORTS", "c_uint16"]
