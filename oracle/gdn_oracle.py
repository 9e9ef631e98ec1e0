"""CPU oracle for the GDN decode and prefill operators — TEST INFRASTRUCTURE ONLY.

This module restates, in fp32 PyTorch on the CPU, the reference's own GDN
implementation of the hot path:

* decode:  gdn/decode/baseline/triton/kernel.py:27-100
* prefill: gdn/prefill/baseline/triton/kernel.py:18-100

It is the checker the parity tests, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline leg compare the CUDA kernels against. Nothing in
the product path (``flashinfer_bench_tma_thrust_b200``) may import it.

Parity pin: ``tests/golden/`` holds fixtures produced by running the
reference's own baseline kernels (imported from the reference checkout) on
seeded inputs (``tests/golden/make_golden.py``); ``tests/test_oracle_golden.py``
checks this restatement against every one of them.

The restatement keeps the reference's arithmetic (fp32 throughout, bf16
rounding of the output only) but works directly on the k-last state rows
S[v, :] instead of transposing to k-first: the k-first update
H <- gH + k (x)(beta (v - k^T gH)) is, row by row of S = H^T,
S[v,:] <- g S[v,:] + beta (v_v - g S[v,:].k) k.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def _scale(scale, head_dim: int) -> float:
    # gdn/decode/baseline/triton/kernel.py:52-53, gdn/prefill/baseline/triton/kernel.py:46-47
    if scale is None:
        return 1.0 / math.sqrt(head_dim)
    scale = float(scale)
    return 1.0 / math.sqrt(head_dim) if scale == 0.0 else scale


def gates(A_log, a, dt_bias, b):
    """g = exp(-exp(A_log) softplus(a + dt_bias)), beta = sigmoid(b), all fp32.

    gdn/decode/baseline/triton/kernel.py:57-59 (torch softplus: threshold 20).
    Shapes broadcast: A_log/dt_bias [HV], a/b [..., HV].
    """
    x = a.float() + dt_bias.float()
    g = torch.exp(-torch.exp(A_log.float()) * F.softplus(x))
    beta = torch.sigmoid(b.float())
    return g, beta


def _step(S, q, k, v, g, beta, scale):
    """One recurrent step for a batch of heads, k-last rows.

    S [..., V, K] fp32 (updated copy returned), q/k [..., K], v [..., V],
    g/beta [...]. Returns (o [..., V] fp32, S_new).
    Reference token step: gdn/prefill/baseline/triton/kernel.py:83-95.
    """
    Sg = g[..., None, None] * S                                  # decay
    old = torch.einsum("...vk,...k->...v", Sg, k)                 # S k  (old_v)
    delta = beta[..., None] * (v - old)                           # new_v - old_v
    S_new = Sg + delta[..., :, None] * k[..., None, :]            # rank-1 delta rule
    o = scale * torch.einsum("...vk,...k->...v", S_new, q)        # readout
    return o, S_new


@torch.no_grad()
def decode(q, k, v, state, A_log, a, dt_bias, b, scale=None):
    """Oracle of gdn/decode/baseline/triton/kernel.py:27-100.

    q,k [B,1,HQ,D] bf16; v [B,1,HV,D]; state [B,HV,D,D] fp32 k-last or None.
    Returns (output [B,1,HV,D] bf16, new_state [B,HV,D,D] fp32 contiguous).
    """
    B, T, HQ, D = q.shape
    HV = v.shape[2]
    assert T == 1
    scale = _scale(scale, D)
    g, beta = gates(A_log, a, dt_bias, b)                    # [B,1,HV]
    ratio = HV // HQ                                         # kernel.py:69-71 GVA expansion
    qf = q.float()[:, 0].repeat_interleave(ratio, dim=1)     # [B,HV,D]
    kf = k.float()[:, 0].repeat_interleave(ratio, dim=1)
    vf = v.float()[:, 0]
    S = state.float() if state is not None else torch.zeros(B, HV, D, D)
    o, S_new = _step(S, qf, kf, vf, g[:, 0], beta[:, 0], scale)
    return o.unsqueeze(1).to(torch.bfloat16), S_new.contiguous()


@torch.no_grad()
def prefill(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale=None):
    """Oracle of gdn/prefill/baseline/triton/kernel.py:18-100 (per-token loop).

    q,k [T,HQ,D] bf16; v [T,HV,D]; a,b [T,HV]; cu_seqlens [N+1] int32/int64;
    state [N,HV,D,D] fp32 k-last or None.
    Returns (output [T,HV,D] bf16, new_state [N,HV,D,D] fp32).
    """
    T, HQ, D = q.shape
    HV = v.shape[1]
    N = cu_seqlens.numel() - 1
    scale = _scale(scale, D)
    g, beta = gates(A_log, a, dt_bias, b)                    # [T,HV]
    ratio = HV // HQ
    qf = q.float().repeat_interleave(ratio, dim=1)           # [T,HV,D]
    kf = k.float().repeat_interleave(ratio, dim=1)
    vf = v.float()
    out = torch.zeros(T, HV, D, dtype=torch.bfloat16)
    new_state = torch.zeros(N, HV, D, D, dtype=torch.float32)
    cu = [int(x) for x in cu_seqlens.tolist()]
    for n in range(N):
        start, end = cu[n], cu[n + 1]
        if end - start <= 0:                                 # kernel.py:68-71 passthrough
            if state is not None:
                new_state[n] = state[n].float()
            continue
        S = state[n].float().clone() if state is not None else torch.zeros(HV, D, D)
        for t in range(start, end):
            o, S = _step(S, qf[t], kf[t], vf[t], g[t], beta[t], scale)
            out[t] = o.to(torch.bfloat16)
        new_state[n] = S
    return out, new_state
