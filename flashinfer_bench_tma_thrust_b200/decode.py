"""GDN single-token decode — drop-in for the reference's decode solution entry.

``kernel(q, k, v, state, A_log, a, dt_bias, b, scale) -> (output, new_state)``
has the signature of ``gdn/decode/solution/triton/kernel.py:85`` (selected by
``gdn/decode/config.toml``: ``entry_point = "kernel.py::kernel"``) and the tensor
contract of ``gdn/trace_definitions/gdn_decode_qk4_v8_d128_k_last.json``:

    q, k     [B, 1, HQ, 128] bf16        v [B, 1, HV, 128] bf16
    state    [B, HV, 128, 128] fp32 k-last, or None (zeros)
    A_log    [HV] fp32    a [B, 1, HV] bf16/fp32    dt_bias [HV] fp32    b [B, 1, HV]
    scale    float, None or 0.0 -> 1/sqrt(128)
    returns  output [B, 1, HV, 128] bf16, new_state [B, HV, 128, 128] fp32

Inputs are never modified (the reference clones the state,
gdn/decode/baseline/triton/kernel.py:75). ``kernel_inplace`` is the
serving-oriented variant that writes the new state over ``state``.
All work runs in one launch of the sm_100a decode kernel on the current stream.
"""
from __future__ import annotations

import torch

from . import _checks as C
from . import _lib


def _launch(q, k, v, state, A_log, a, dt_bias, b, scale, out, new_state):
    dev = q.device
    B, T, HQ, D = q.shape
    if T != 1:
        raise ValueError(f"decode expects seq_len 1 (q.shape[1]), got {T}")
    HV = v.shape[2]
    C.check_heads(HQ, HV, D)
    if k.shape != q.shape:
        raise ValueError(f"k shape {tuple(k.shape)} != q shape {tuple(q.shape)}")
    if tuple(v.shape) != (B, 1, HV, D):
        raise ValueError(f"v must be [B,1,HV,{D}], got {tuple(v.shape)}")
    for name, t in (("q", q), ("k", k), ("v", v), ("A_log", A_log), ("a", a),
                    ("dt_bias", dt_bias), ("b", b)):
        C.require_cuda(name, t, dev)
    if a.numel() != B * HV or b.numel() != B * HV:
        raise ValueError("a and b must have B*HV elements ([B,1,HV])")
    if A_log.numel() != HV or dt_bias.numel() != HV:
        raise ValueError("A_log and dt_bias must have HV elements")
    q_c, k_c, v_c = C.as_bf16("q", q), C.as_bf16("k", k), C.as_bf16("v", v)
    A_c, A_t = C.as_gate("A_log", A_log)
    a_c, a_t = C.as_gate("a", a)
    d_c, d_t = C.as_gate("dt_bias", dt_bias)
    b_c, b_t = C.as_gate("b", b)
    s_c = None
    if state is not None:
        C.require_cuda("state", state, dev)
        if tuple(state.shape) != (B, HV, D, D):
            raise ValueError(f"state must be [B,HV,{D},{D}], got {tuple(state.shape)}")
        s_c = state.float().contiguous()
    lib = _lib.load()
    with torch.cuda.device(dev):
        rc = lib.gdn_decode_fwd(
            q_c.data_ptr(), k_c.data_ptr(), v_c.data_ptr(), C.ptr(s_c),
            A_c.data_ptr(), A_t, a_c.data_ptr(), a_t, d_c.data_ptr(), d_t, b_c.data_ptr(), b_t,
            C.resolve_scale(scale, D), out.data_ptr(), new_state.data_ptr(), B, HQ, HV, D,
            C.stream_handle(dev))
    _lib.check(rc, "gdn_decode_fwd")
    return out, new_state


def kernel(q, k, v, state, A_log, a, dt_bias, b, scale=None):
    """Reference-compatible decode: returns freshly allocated (output, new_state)."""
    B, _, _, D = q.shape
    HV = v.shape[2]
    out = torch.empty(B, 1, HV, D, dtype=torch.bfloat16, device=q.device)
    new_state = torch.empty(B, HV, D, D, dtype=torch.float32, device=q.device)
    return _launch(q, k, v, state, A_log, a, dt_bias, b, scale, out, new_state)


def kernel_inplace(q, k, v, state, A_log, a, dt_bias, b, scale=None, out=None):
    """Decode that updates ``state`` (fp32, contiguous) in place; returns (output, state)."""
    if state is None or state.dtype != torch.float32 or not state.is_contiguous():
        raise ValueError("kernel_inplace needs a contiguous fp32 state tensor")
    B, _, _, D = q.shape
    HV = v.shape[2]
    if out is None:
        out = torch.empty(B, 1, HV, D, dtype=torch.bfloat16, device=q.device)
    return _launch(q, k, v, state, A_log, a, dt_bias, b, scale, out, state)


def kernel_bf16_state(q, k, v, state, A_log, a, dt_bias, b, scale=None, out=None,
                      new_state=None):
    """Reduced-precision option: decode with a bf16 state [B, HV, 128, 128] (k-last).
    fp32 math, new state rounded to bf16 — half the HBM bytes of the fp32 path, with
    its own error (see tests/test_decode_bf16_state_gpu.py). ``new_state`` may be the
    input ``state`` (in place). Returns (output bf16 [B,1,HV,128], new_state bf16)."""
    dev = q.device
    B, T, HQ, D = q.shape
    if T != 1:
        raise ValueError(f"decode expects seq_len 1 (q.shape[1]), got {T}")
    HV = v.shape[2]
    C.check_heads(HQ, HV, D)
    for name, t in (("q", q), ("k", k), ("v", v), ("A_log", A_log), ("a", a),
                    ("dt_bias", dt_bias), ("b", b)):
        C.require_cuda(name, t, dev)
    if state is not None:
        C.require_cuda("state", state, dev)
        if state.dtype != torch.bfloat16 or tuple(state.shape) != (B, HV, D, D):
            raise ValueError("state must be bf16 [B, HV, 128, 128]")
        state = state.contiguous()
    q_c, k_c, v_c = C.as_bf16("q", q), C.as_bf16("k", k), C.as_bf16("v", v)
    A_c, A_t = C.as_gate("A_log", A_log)
    a_c, a_t = C.as_gate("a", a)
    d_c, d_t = C.as_gate("dt_bias", dt_bias)
    b_c, b_t = C.as_gate("b", b)
    if out is None:
        out = torch.empty(B, 1, HV, D, dtype=torch.bfloat16, device=dev)
    if new_state is None:
        new_state = torch.empty(B, HV, D, D, dtype=torch.bfloat16, device=dev)
    lib = _lib.load()
    with torch.cuda.device(dev):
        rc = lib.gdn_decode_fwd_bf16state(
            q_c.data_ptr(), k_c.data_ptr(), v_c.data_ptr(), C.ptr(state),
            A_c.data_ptr(), A_t, a_c.data_ptr(), a_t, d_c.data_ptr(), d_t, b_c.data_ptr(), b_t,
            C.resolve_scale(scale, D), out.data_ptr(), new_state.data_ptr(), B, HQ, HV, D,
            C.stream_handle(dev))
    _lib.check(rc, "gdn_decode_fwd_bf16state")
    return out, new_state


def kernel_multitoken(q, k, v, state, A_log, a, dt_bias, b, scale=None):
    """Decode T >= 1 tokens per sequence in one call (speculative / multi-token decode).

    Shapes as ``kernel`` with T = q.shape[1] tokens per sequence: q, k [B,T,HQ,128],
    v [B,T,HV,128], a, b [B,T,HV]. The B sequences are equal-length segments of one
    chunked prefill (cu_seqlens = 0, T, 2T, ...), so the result is the same as T
    consecutive ``kernel`` calls. Returns (output [B,T,HV,128] bf16, new_state fp32).
    """
    from . import prefill
    B, T, HQ, D = q.shape
    HV = v.shape[2]
    if T == 1:
        return kernel(q, k, v, state, A_log, a, dt_bias, b, scale)
    cu = torch.arange(0, (B + 1) * T, T, dtype=torch.int64, device=q.device)
    out, new_state = prefill.kernel(q.reshape(B * T, HQ, D), k.reshape(B * T, HQ, D),
                                    v.reshape(B * T, HV, D), state, A_log,
                                    a.reshape(B * T, HV), dt_bias, b.reshape(B * T, HV), cu,
                                    scale)
    return out.view(B, T, HV, D), new_state


def quantize_state_fp8(state: torch.Tensor):
    """fp32 state [..., V, K] -> (E4M3 codes as uint8, fp32 per-row scales [..., V]),
    the layout of ``kernel_fp8_state`` (scale = max|row| / 448)."""
    s = state.float()
    amax = s.abs().amax(dim=-1)
    scale = torch.where(amax > 0, amax / 448.0, torch.ones_like(amax))
    codes = (s / scale[..., None]).to(torch.float8_e4m3fn).view(torch.uint8)
    return codes, scale


def dequantize_state_fp8(codes: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    return codes.view(torch.float8_e4m3fn).float() * scale[..., None]


def kernel_fp8_state(q, k, v, state_codes, state_scale, A_log, a, dt_bias, b, scale=None):
    """Reduced-precision option: decode with an FP8 E4M3 state (uint8 codes
    [B, HV, 128, 128] + fp32 per-row scales [B, HV, 128]). fp32 math; the new state is
    requantised per row. ~3.9x fewer state bytes than fp32, with its own error (see
    tests/test_decode_fp8_state_gpu.py). Returns (output, new_codes, new_scales)."""
    dev = q.device
    B, T, HQ, D = q.shape
    if T != 1:
        raise ValueError(f"decode expects seq_len 1 (q.shape[1]), got {T}")
    HV = v.shape[2]
    C.check_heads(HQ, HV, D)
    for name, t in (("q", q), ("k", k), ("v", v), ("A_log", A_log), ("a", a),
                    ("dt_bias", dt_bias), ("b", b)):
        C.require_cuda(name, t, dev)
    if state_codes is not None:
        if state_codes.dtype != torch.uint8 or tuple(state_codes.shape) != (B, HV, D, D):
            raise ValueError("state codes must be uint8 [B, HV, 128, 128]")
        if state_scale is None or tuple(state_scale.shape) != (B, HV, D):
            raise ValueError("state scales must be fp32 [B, HV, 128]")
        state_codes = state_codes.contiguous()
        state_scale = state_scale.float().contiguous()
    q_c, k_c, v_c = C.as_bf16("q", q), C.as_bf16("k", k), C.as_bf16("v", v)
    A_c, A_t = C.as_gate("A_log", A_log)
    a_c, a_t = C.as_gate("a", a)
    d_c, d_t = C.as_gate("dt_bias", dt_bias)
    b_c, b_t = C.as_gate("b", b)
    out = torch.empty(B, 1, HV, D, dtype=torch.bfloat16, device=dev)
    new_codes = torch.empty(B, HV, D, D, dtype=torch.uint8, device=dev)
    new_scale = torch.empty(B, HV, D, dtype=torch.float32, device=dev)
    lib = _lib.load()
    with torch.cuda.device(dev):
        rc = lib.gdn_decode_fwd_fp8state(
            q_c.data_ptr(), k_c.data_ptr(), v_c.data_ptr(), C.ptr(state_codes),
            C.ptr(state_scale), A_c.data_ptr(), A_t, a_c.data_ptr(), a_t, d_c.data_ptr(), d_t,
            b_c.data_ptr(), b_t, C.resolve_scale(scale, D), out.data_ptr(), new_codes.data_ptr(),
            new_scale.data_ptr(), B, HQ, HV, D, C.stream_handle(dev))
    _lib.check(rc, "gdn_decode_fwd_fp8state")
    return out, new_codes, new_scale
