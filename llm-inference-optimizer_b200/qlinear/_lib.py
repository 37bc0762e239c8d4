"""ctypes binding of libqlinear.so (C ABI declared in include/qlinear.h).

The shared library is built in-tree (``python -m qlinear._build``) and
loaded from this directory.  There is no fallback: if the library is
missing, every kernel entry point raises instead of silently running
something else.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

LIB_NAME = "libqlinear.so"
LIB_PATH = Path(__file__).resolve().parent / LIB_NAME

# status codes (include/qlinear.h)
QL_OK = 0
QL_ERR_NULL_POINTER = -1
QL_ERR_BAD_SHAPE = -2
QL_ERR_BAD_STRIDE = -3
QL_ERR_UNSUPPORTED = -4
QL_ERR_WORKSPACE = -5
QL_ERR_CUDA = -6
QL_ERR_DEVICE = -7
QL_ERR_DEVICE_TIMEOUT = -8

QL_DTYPE_F16 = 0
QL_DTYPE_F32 = 1
QL_DTYPE_BF16 = 2

QL_STATIC_WS_BYTES = 2 * 1024 * 1024

QL_DEVICE_ERROR_FULL_WAIT = 1
QL_DEVICE_ERROR_EMPTY_WAIT = 2
QL_DEVICE_ERROR_MMA_WAIT = 3
QL_DEVICE_ERROR_TMEM = 4
QL_DEVICE_ERROR_PEER_WAIT = 5
QL_XCHG_MAX_RANKS = 8

QL_W4_LAYOUT_SPLIT_HALF = 0
QL_W4_LAYOUT_ADJACENT = 1

QL_FLAG_PDL = 0x1
QL_FLAG_FORCE_GEMM = 0x2
QL_FLAG_FORCE_GEMV = 0x4
QL_FLAG_FORCE_GENERIC = 0x8
QL_FLAG_FORCE_TCDEC = 0x10

_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int
_sz = ctypes.c_size_t
_uint = ctypes.c_uint

# name -> (restype, argtypes)
SIGNATURES = {
    "ql_w8a16_linear": (_int, [_vp, _int, _vp, _vp, _int, _vp, _int, _vp,
                               _i64, _i64, _i64, _i64, _i64, _i64, _vp, _sz, _uint, _vp]),
    "ql_w4a16_linear": (_int, [_vp, _int, _vp, _int, _vp, _vp, _int, _vp,
                               _i64, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _sz, _uint, _vp]),
    "ql_w4a16_linear_static_ws": (_int, [_vp, _int, _vp, _int, _vp, _vp, _int, _vp,
                                         _i64, _i64, _i64, _i64, _i64, _i64, _i64, _uint, _vp]),
    "ql_w8a16_gate_up_silu": (_int, [_vp, _int, _vp, _vp, _int, _vp, _int, _vp,
                                     _i64, _i64, _i64, _i64, _i64, _i64, _vp, _sz, _uint, _vp]),
    "ql_w4a16_gate_up_silu": (_int, [_vp, _int, _vp, _int, _vp, _vp, _int, _vp,
                                     _i64, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _sz, _uint, _vp]),
    "ql_w8a16_gate_up_silu_workspace_size": (_sz, [_i64, _i64, _i64]),
    "ql_w4a16_gate_up_silu_workspace_size": (_sz, [_i64, _i64, _i64]),
    "ql_w8a16_workspace_size": (_sz, [_i64, _i64, _i64]),
    "ql_w4a16_workspace_size": (_sz, [_i64, _i64, _i64]),
    "ql_gemv_plan": (_int, [_int, _i64, _i64, _i64, _sz, ctypes.POINTER(_i64), _int]),
    "ql_gemm_plan": (_int, [_int, _int, _i64, _i64, _i64, ctypes.POINTER(_i64), _int]),
    "ql_tcdec_plan": (_int, [_int, _i64, _i64, _i64, ctypes.POINTER(_i64), _int]),
    "ql_w8a16_dequantize": (_int, [_vp, _vp, _int, _vp, _i64, _i64, _i64, _vp]),
    "ql_w4a16_dequantize": (_int, [_vp, _int, _vp, _vp, _i64, _i64, _i64, _i64, _vp]),
    "ql_w4a16_unpack": (_int, [_vp, _int, _vp, _i64, _i64, _i64, _vp]),
    "ql_w8a16_quantize": (_int, [_vp, _i64, _i64, _i64, _vp, _vp, _vp]),
    "ql_w4a16_quantize": (_int, [_vp, _i64, _i64, _i64, _int, _int, _vp, _vp, _vp]),
    "ql_argmax_rows_f16": (_int, [_vp, _i64, _i64, _i64, _i64, _vp, _vp]),
    "ql_xchg_buffer_bytes": (_sz, [_int, _int]),
    "ql_xchg_alloc": (_int, [_sz, ctypes.POINTER(_vp), _vp]),
    "ql_xchg_free": (_int, [_vp]),
    "ql_xchg_open": (_int, [_vp, ctypes.POINTER(_vp)]),
    "ql_xchg_close": (_int, [_vp]),
    "ql_argmax_exchange_f16": (_int, [_vp, _i64, _i64, _i64, _i64, _int, _int, _int, ctypes.POINTER(_vp), _vp,
                                      _vp]),
    "ql_w8a16_linear_argmax": (_int, [_vp, _int, _vp, _vp, _int, _vp, _int, _i64, _i64, _i64, _i64, _i64,
                                      _i64, _int, _int, _int, ctypes.POINTER(_vp), _vp, _uint, _vp]),
    "ql_w4a16_linear_argmax": (_int, [_vp, _int, _vp, _int, _vp, _vp, _int, _i64, _i64, _i64, _i64, _i64,
                                      _i64, _i64, _int, _int, _int, ctypes.POINTER(_vp), _vp, _uint, _vp]),
    "ql_linear_argmax_supported": (_int, [_int, _i64, _i64, _i64]),
    "ql_gather_buffer_bytes": (_sz, [_int, _i64]),
    "ql_allgather_f16": (_int, [_vp, _i64, _vp, _i64, _i64, _i64, _int, _i64, _int, _int, _int,
                                ctypes.POINTER(_vp), _uint, _vp]),
    "ql_strerror": (ctypes.c_char_p, [_int]),
    "ql_version": (_int, []),
    "ql_device_error": (_int, [ctypes.POINTER(_int)]),
    "ql_clear_device_error": (_int, []),
}

_lock = threading.Lock()
_lib = None


class QLinearError(RuntimeError):
    """A libqlinear entry point returned a non-zero status."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


def load(path: Path | str | None = None) -> ctypes.CDLL:
    """Load (once) and return the library with typed entry points."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = Path(path) if path is not None else Path(os.environ.get("QLINEAR_LIB", LIB_PATH))
        if not p.exists():
            raise ImportError(
                f"{LIB_NAME} is not built ({p} missing). Build it with "
                "`python -m qlinear._build` (nvcc, sm_100a); this package has no "
                "fallback implementation.")
        lib = ctypes.CDLL(str(p))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if path is None:
            _lib = lib
        return lib


def check(status: int) -> None:
    if status != QL_OK:
        msg = load().ql_strerror(status)
        raise QLinearError(status, (msg or b"qlinear: error").decode())


PLAN_FIELDS = ("tiles_per_cta", "warps_per_tile", "k_splits", "kblocks_per_split", "stages",
               "batch_tiles", "batch_chunks", "ctas", "smem_bytes", "workspace_bytes", "kblocks_per_stage",
               "chunk_bytes", "cost_ns")


def gemv_plan(wbits: int, M: int, N: int, K: int, workspace_bytes: int | None = None) -> dict:
    """The decode-kernel plan for a shape (see ql_gemv_plan)."""
    buf = (_i64 * 13)()
    avail = (1 << 64) - 1 if workspace_bytes is None else workspace_bytes
    check(load().ql_gemv_plan(wbits, M, N, K, avail, buf, 13))
    return dict(zip(PLAN_FIELDS, list(buf)))


GEMM_PLAN_FIELDS = ("rows_per_tile", "k_splits", "stages_per_split", "ring_stages", "smem_bytes", "tiles",
                    "ctas", "clusters_fit")


def gemm_plan(wbits: int, M: int, N: int, K: int, layout: int = QL_W4_LAYOUT_SPLIT_HALF) -> dict:
    """The tensor-core kernel's launch plan for a shape (see ql_gemm_plan)."""
    buf = (_i64 * 8)()
    check(load().ql_gemm_plan(wbits, layout, M, N, K, buf, 8))
    return dict(zip(GEMM_PLAN_FIELDS, list(buf)))


TCDEC_PLAN_FIELDS = ("rows_per_tile", "k_splits", "blocks_per_split", "stages", "smem_bytes", "tiles",
                     "dispatched")


def tcdec_plan(wbits: int, M: int, N: int, K: int) -> dict | None:
    """The small-batch tensor-core kernel's plan for a shape (see
    ql_tcdec_plan); None where the kernel cannot take it."""
    buf = (_i64 * 7)()
    st = load().ql_tcdec_plan(wbits, M, N, K, buf, 7)
    if st == QL_ERR_UNSUPPORTED:
        return None
    check(st)
    return dict(zip(TCDEC_PLAN_FIELDS, list(buf)))


def version() -> tuple[int, int, int]:
    v = load().ql_version()
    return (v >> 16) & 0xFF, (v >> 8) & 0xFF, v & 0xFF


def device_error() -> int:
    """Reads the device error word (synchronises the device)."""
    code = _int(0)
    check(load().ql_device_error(ctypes.byref(code)))
    return code.value


def clear_device_error() -> None:
    check(load().ql_clear_device_error())
