"""B200-native (sm_100a) Gated Delta Net decode and prefill operators.

Drop-in replacements for the solution entry points of the reference's GDN
operators (gdn/decode/solution/*/kernel.py, gdn/prefill/solution/*/kernel.py):

    from flashinfer_bench_tma_thrust_b200 import decode, prefill
    out, new_state = decode.kernel(q, k, v, state, A_log, a, dt_bias, b, scale)
    out, new_state = prefill.kernel(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale)

The compute runs in ``libgdn_b200.so`` (hand-written CUDA for sm_100a behind a
C ABI, ``include/gdn_b200.h``); PyTorch only provides device memory and streams.
"""
from . import decode, prefill  # noqa: F401
from ._lib import GDNError  # noqa: F401

__all__ = ["decode", "prefill", "GDNError"]
