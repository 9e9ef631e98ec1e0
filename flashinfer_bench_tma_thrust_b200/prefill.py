"""GDN variable-length prefill — drop-in for the reference's prefill solution entry.

``kernel(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale) -> (output, new_state)``
has the signature of ``gdn/prefill/solution/triton/kernel.py:272`` (selected by
``gdn/prefill/config.toml``) and the tensor contract of
``gdn/trace_definitions/gdn_prefill_qk4_v8_d128_k_last.json``:

    q, k        [T, HQ, 128] bf16          v [T, HV, 128] bf16
    state       [N, HV, 128, 128] fp32 k-last, or None (zeros)
    A_log       [HV] fp32    a, b [T, HV] bf16/fp32    dt_bias [HV] fp32
    cu_seqlens  [N+1] int64 (definition) or int32 (reference tests)
    returns     output [T, HV, 128] bf16, new_state [N, HV, 128, 128] fp32

A sequence with cu_seqlens[n+1] <= cu_seqlens[n] passes its state through
(gdn/prefill/baseline/triton/kernel.py:68-71). Inputs are never modified.

``kernel_recurrent`` runs the token-sequential kernel (the independent
cross-check); ``kernel`` runs the chunked tensor-core kernel.
"""
from __future__ import annotations

import torch

from . import _checks as C
from . import _lib


class _Prepared:
    __slots__ = ("dev", "T", "N", "HQ", "HV", "D", "q", "k", "v", "state", "A", "A_t", "a",
                 "a_t", "d", "d_t", "b", "b_t", "cu", "cu_t", "scale")


def prepare(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale) -> _Prepared:
    """Validate shapes/dtypes/devices and make every tensor contiguous."""
    P = _Prepared()
    dev = q.device
    if q.dim() != 3:
        raise ValueError(f"q must be [T, HQ, D], got {tuple(q.shape)}")
    T, HQ, D = q.shape
    if v.dim() != 3 or v.shape[0] != T or v.shape[2] != D:
        raise ValueError(f"v must be [T, HV, {D}], got {tuple(v.shape)}")
    HV = v.shape[1]
    C.check_heads(HQ, HV, D)
    if k.shape != q.shape:
        raise ValueError(f"k shape {tuple(k.shape)} != q shape {tuple(q.shape)}")
    for name, t in (("q", q), ("k", k), ("v", v), ("A_log", A_log), ("a", a),
                    ("dt_bias", dt_bias), ("b", b), ("cu_seqlens", cu_seqlens)):
        C.require_cuda(name, t, dev)
    if cu_seqlens.dim() != 1 or cu_seqlens.numel() < 1:
        raise ValueError("cu_seqlens must be a 1-D tensor of length num_seqs + 1")
    N = cu_seqlens.numel() - 1
    if a.numel() != T * HV or b.numel() != T * HV:
        raise ValueError("a and b must be [T, HV]")
    if A_log.numel() != HV or dt_bias.numel() != HV:
        raise ValueError("A_log and dt_bias must have HV elements")
    P.dev, P.T, P.N, P.HQ, P.HV, P.D = dev, T, N, HQ, HV, D
    P.q, P.k, P.v = C.as_bf16("q", q), C.as_bf16("k", k), C.as_bf16("v", v)
    P.A, P.A_t = C.as_gate("A_log", A_log)
    P.a, P.a_t = C.as_gate("a", a)
    P.d, P.d_t = C.as_gate("dt_bias", dt_bias)
    P.b, P.b_t = C.as_gate("b", b)
    P.cu, P.cu_t = C.as_index("cu_seqlens", cu_seqlens)
    P.state = None
    if state is not None:
        C.require_cuda("state", state, dev)
        if tuple(state.shape) != (N, HV, D, D):
            raise ValueError(f"state must be [N,HV,{D},{D}], got {tuple(state.shape)}")
        P.state = state.float().contiguous()
    P.scale = C.resolve_scale(scale, D)
    return P


def _alloc_outputs(P: _Prepared):
    out = torch.empty(P.T, P.HV, P.D, dtype=torch.bfloat16, device=P.dev)
    new_state = torch.empty(P.N, P.HV, P.D, P.D, dtype=torch.float32, device=P.dev)
    return out, new_state


def _ptr0(t):
    # zero-element tensors may report a null data_ptr; the ABI accepts that when T == 0
    return t.data_ptr() if t.numel() else None


def run_recurrent(P: _Prepared, out, new_state):
    lib = _lib.load()
    with torch.cuda.device(P.dev):
        rc = lib.gdn_prefill_recurrent_fwd(
            _ptr0(P.q), _ptr0(P.k), _ptr0(P.v), C.ptr(P.state),
            P.A.data_ptr(), P.A_t, _ptr0(P.a), P.a_t, P.d.data_ptr(), P.d_t, _ptr0(P.b), P.b_t,
            P.cu.data_ptr(), P.cu_t, P.scale, _ptr0(out), _ptr0(new_state),
            P.T, P.N, P.HQ, P.HV, P.D, C.stream_handle(P.dev))
    _lib.check(rc, "gdn_prefill_recurrent_fwd")
    return out, new_state


def kernel_recurrent(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale=None):
    """Token-sequential prefill (one launch of the SIMT recurrent kernel)."""
    P = prepare(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale)
    out, new_state = _alloc_outputs(P)
    return run_recurrent(P, out, new_state)


_workspaces: dict = {}
# per device: (pinned host int32 copy of the status word, event recorded after the copy)
_status_probe: dict = {}


def workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """Per-device workspace of the chunked prefill (zeroed once; its first bytes hold
    the sticky status word, the rest the per-chunk units of the two-phase path: the
    [T_b; P] operand image and the chunk's gates, 24.5 KB per (chunk, v-head)). Grown on
    demand, never shrunk; a grown workspace keeps the status bits set so far. Calls on
    one device share it, so they must be ordered on one stream."""
    key = (device.type, device.index)
    ws = _workspaces.get(key)
    if ws is None or ws.numel() < nbytes:
        new = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=device)
        if ws is not None:
            new[:4].copy_(ws[:4])  # stream-ordered: the sticky bits survive the growth
        ws = new
        _workspaces[key] = ws
    return ws


def _device_key(device):
    device = torch.device(device or torch.cuda.current_device())
    if device.type == "cuda" and device.index is None:
        device = torch.device("cuda", torch.cuda.current_device())
    return (device.type, device.index)


def device_status(device=None) -> int:
    """Sticky status word of the chunked kernel on `device`, a bit set: 0 = clean;
    bit 0 (1) = a bounded wait gave up (outputs of that call invalid); bit 1 (2) =
    cu_seqlens held a value outside [0, T] (used clamped) or overlapping ranges whose
    chunks overflow the workspace (that call computed nothing and passed states
    through). Synchronises."""
    ws = _workspaces.get(_device_key(device))
    if ws is None:
        return 0
    return int(ws[:4].view(torch.int32).item())


def reset_device_status(device=None) -> None:
    """Clear the sticky status word on `device` (stream-ordered on the current stream) and
    the host copy that the next call checks."""
    key = _device_key(device)
    ws = _workspaces.get(key)
    if ws is not None:
        ws[:4].zero_()
    probe = _status_probe.get(key)
    if probe is not None:
        probe[1].synchronize()
        probe[0].zero_()


def _aligned(t):
    return t if t.numel() == 0 or t.data_ptr() % 16 == 0 else t.clone()


_FUSED_WORKSPACE_BYTES = 256


def run_chunked(P: _Prepared, out, new_state, fused: bool = False):
    """Chunked tensor-core prefill. With the full workspace the C library runs the
    two-phase path (parallel prep of the per-chunk [T_b; P] operands, then the state
    scan); ``fused=True`` hands it only 256 bytes, which selects the single-kernel path."""
    lib = _lib.load()
    q, k, v = _aligned(P.q), _aligned(P.k), _aligned(P.v)
    if fused:
        ws = workspace(P.dev, _FUSED_WORKSPACE_BYTES)
        nbytes = _FUSED_WORKSPACE_BYTES
    else:
        nbytes = lib.gdn_prefill_chunked_workspace_size(P.T, P.N, P.HV)
        ws = workspace(P.dev, nbytes)
    with torch.cuda.device(P.dev):
        rc = lib.gdn_prefill_chunked_fwd(
            _ptr0(q), _ptr0(k), _ptr0(v), C.ptr(P.state),
            P.A.data_ptr(), P.A_t, _ptr0(P.a), P.a_t, P.d.data_ptr(), P.d_t, _ptr0(P.b), P.b_t,
            P.cu.data_ptr(), P.cu_t, P.scale, _ptr0(out), _ptr0(new_state),
            P.T, P.N, P.HQ, P.HV, P.D, ws.data_ptr(), nbytes, C.stream_handle(P.dev))
    _lib.check(rc, "gdn_prefill_chunked_fwd")
    return out, new_state


def _check_status(dev, check: bool) -> None:
    """Report a failure of a chunked call on `dev`. Every call queues an asynchronous copy
    of the sticky status word into pinned host memory; the next call on the device reads
    the copy if it has landed (no synchronisation) and raises GDNError for any bit set.
    With check=True the call waits for its own copy and raises for its own failure."""
    key = (dev.type, dev.index)
    probe = _status_probe.get(key)
    if probe is not None and (check or probe[1].query()):
        if check:
            probe[1].synchronize()
        st = int(probe[0].item())
        if st:
            raise _lib.GDNError(
                f"gdn_prefill_chunked_fwd reported status bits {st:#x} on {dev} "
                "(1: a bounded wait gave up; 2: invalid cu_seqlens); the outputs of the "
                "failing call are invalid. Clear with reset_device_status().")


def _queue_status_copy(dev) -> None:
    key = (dev.type, dev.index)
    probe = _status_probe.get(key)
    if probe is None:
        probe = (torch.zeros(1, dtype=torch.int32).pin_memory(), torch.cuda.Event())
        _status_probe[key] = probe
    ws = _workspaces[key]
    probe[0].copy_(ws[:4].view(torch.int32), non_blocking=True)
    probe[1].record()


def kernel(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale=None, *, check=False):
    """Reference-compatible prefill entry point: one call of the chunked tensor-core
    kernel (chunk 64, state carried in fp32). A failure that the kernels report through
    the device status word (a bounded wait that gave up, invalid cu_seqlens) raises
    GDNError at the next call on the device, or at this call with ``check=True``
    (which synchronises on the status copy)."""
    P = prepare(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale)
    _check_status(P.dev, False)
    out, new_state = _alloc_outputs(P)
    run_chunked(P, out, new_state)
    with torch.cuda.device(P.dev):
        _queue_status_copy(P.dev)
    if check:
        _check_status(P.dev, True)
    return out, new_state


def kernel_fused(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale=None):
    """Chunked prefill on the single-kernel path (needs only a 256-byte workspace)."""
    P = prepare(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale)
    out, new_state = _alloc_outputs(P)
    return run_chunked(P, out, new_state, fused=True)


def launches_per_call(n_seqs: int = 1, T: int = 0, HV: int = 32) -> int:
    """Kernel launches one ``kernel()`` call over ``n_seqs`` sequences of ``T`` tokens in
    total makes on the current device, as the library reports it
    (``gdn_prefill_chunked_launches``): chunk offsets (with the scan order up to 1024
    sequences), chunk gates, prep, scan; a separate scan-order launch above 1024
    sequences; a second prep and scan when the call is split."""
    lib = _lib.load()
    ws = lib.gdn_prefill_chunked_workspace_size(T, n_seqs, HV)
    n = lib.gdn_prefill_chunked_launches(T, n_seqs, HV, ws)
    _lib.check(n if n < 0 else 0, "gdn_prefill_chunked_launches")
    return n
