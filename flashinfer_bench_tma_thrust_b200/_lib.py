"""ctypes binding of ``libgdn_b200.so`` (the C ABI in ``include/gdn_b200.h``).

The library is loaded from this package directory. There is no fallback: if
the library is missing or fails to load, every operator raises, so a GPU box
without the CUDA build can never silently run something else.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_NAME = "libgdn_b200.so"
LIB_PATH = Path(__file__).resolve().parent / LIB_NAME

GDN_OK = 0
DTYPE_F32, DTYPE_BF16, DTYPE_I32, DTYPE_I64 = 0, 1, 2, 3

_p = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_f32 = ctypes.c_float
_int = ctypes.c_int
_size = ctypes.c_size_t

# name -> (restype, argtypes); mirrors include/gdn_b200.h
SIGNATURES = {
    "gdn_abi_version": (_int, []),
    "gdn_status_string": (ctypes.c_char_p, [_int]),
    "gdn_decode_fwd": (
        _int,
        [_p, _p, _p, _p,  # q k v state
         _p, _int, _p, _int, _p, _int, _p, _int,  # A_log a dt_bias b (+dtype)
         _f32, _p, _p, _i64, _i32, _i32, _i32, _p],
    ),
    "gdn_decode_fwd_bf16state": (
        _int,
        [_p, _p, _p, _p,
         _p, _int, _p, _int, _p, _int, _p, _int,
         _f32, _p, _p, _i64, _i32, _i32, _i32, _p],
    ),
    "gdn_decode_fwd_fp8state": (
        _int,
        [_p, _p, _p, _p, _p,
         _p, _int, _p, _int, _p, _int, _p, _int,
         _f32, _p, _p, _p, _i64, _i32, _i32, _i32, _p],
    ),
    "gdn_prefill_recurrent_fwd": (
        _int,
        [_p, _p, _p, _p,
         _p, _int, _p, _int, _p, _int, _p, _int,
         _p, _int, _f32, _p, _p, _i64, _i64, _i32, _i32, _i32, _p],
    ),
    "gdn_prefill_chunked_workspace_size": (_size, [_i64, _i64, _i32]),
    "gdn_prefill_chunked_fwd": (
        _int,
        [_p, _p, _p, _p,
         _p, _int, _p, _int, _p, _int, _p, _int,
         _p, _int, _f32, _p, _p, _i64, _i64, _i32, _i32, _i32, _p, _size, _p],
    ),
    "gdn_prefill_chunked_status": (_int, [_p, _p, _p]),
    "gdn_prefill_chunked_launches": (_int, [_i64, _i64, _i32, _size]),
    "gdn_prefill_chunked_fwd_noalloc": (
        _int,
        [_p, _p, _p, _p,
         _p, _int, _p, _int, _p, _int, _p, _int,
         _p, _int, _f32, _p, _p, _i64, _i64, _i32, _i32, _i32, _p],
    ),
    "gdn_selftest_umma": (_int, [_p, _p, _p, _int, _int, _p, _p]),
    "gdn_selftest_wait_timeout": (_int, [_p, _p, _p]),
    "gdn_selftest_umma_ts": (_int, [_p, _p, _p, _p, _p]),
}

_lock = threading.Lock()
_lib = None


class GDNError(RuntimeError):
    """A C-ABI call returned a non-zero status."""


def load() -> ctypes.CDLL:
    """Load the library once; raise if it is absent (no fallback path)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise GDNError(
                f"{LIB_NAME} is not built (expected at {LIB_PATH}); run "
                "`python -m flashinfer_bench_tma_thrust_b200.build` or __graft_entry__.build()")
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def check(status: int, what: str) -> None:
    if status != GDN_OK:
        msg = load().gdn_status_string(status).decode()
        raise GDNError(f"{what} failed with status {status}: {msg}")
