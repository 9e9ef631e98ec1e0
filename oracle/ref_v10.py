"""ctypes binding of oracle/_ref/libref_v10.so: the reference's own v10 decode kernels
(gdn/kernels/cute_cpp/gdn_decode_v10.cuh) as a comparator for tests and the bench.
Measurement infrastructure only; the package never imports this."""
from __future__ import annotations

import ctypes
from pathlib import Path

LIB = Path(__file__).resolve().parent / "_ref" / "libref_v10.so"
_lib = None


def available() -> bool:
    return LIB.exists()


def _load():
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(str(LIB))
        p, i, f = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
        _lib.ref_v10_decode.restype = i
        _lib.ref_v10_decode.argtypes = [i, p, p, p, p, p, p, p, p, p, p, f, i, i, i, i, p]
    return _lib


def decode(q, k, v, state, A_log, a, dt_bias, b, out, new_state, scale, block_v, variant=0):
    """One launch of the reference's v10 decode ("cute" = 0, "tma" = 1) on the current
    stream. q/k [B,1,HQ,128], v [B,1,HV,128], a/b [B,1,HV] bf16, A_log/dt_bias fp32,
    state [B,HV,128,128] fp32 (all contiguous); writes out [B,HV,128] bf16 and
    new_state. Returns the CUDA error code of the launch (0 = launched)."""
    import torch
    B, _, HQ, _ = q.shape
    HV = v.shape[2]
    st = torch.cuda.current_stream(q.device).cuda_stream
    return _load().ref_v10_decode(variant, q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                  state.data_ptr(), A_log.data_ptr(), a.data_ptr(),
                                  dt_bias.data_ptr(), b.data_ptr(), out.data_ptr(),
                                  new_state.data_ptr(), float(scale), B, HQ, HV, block_v, st)
