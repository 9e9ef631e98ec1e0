"""CPU model of the chunk-64 prefill algebra the CUDA kernel implements — TEST
INFRASTRUCTURE ONLY (used by tests to show the chunk formulation equals the
reference's per-token recurrence, gdn/prefill/baseline/triton/kernel.py:63-98).

Per sequence, v-head and chunk of C tokens (padded rows: k=q=v=0, beta=0, log g=0),
with H the k-first state [K, V] entering the chunk:

    lg_i = -exp(A_log) softplus(a_i + dt_bias)     Gamma_i = sum_{j<=i} lg_j   gamma_i = exp(Gamma_i)
    A[i,j]  = beta_i exp(Gamma_i - Gamma_j) (k_i . k_j)      j <  i   (else 0)
    M[i,j]  =        exp(Gamma_i - Gamma_j) (q_i . k_j)      j <= i   (else 0)
    T_beta  = (I + A)^-1 diag(beta)                P = M T_beta
    X       = V - diag(gamma) K H                  (K H, Q H: one [K;Q] H product)
    [U; O'] = [T_beta; P] X
    O       = scale (diag(gamma) Q H + O')
    H_next  = gamma_last H + Kt^T U,   Kt_j = exp(Gamma_last - Gamma_j) k_j

This is the chunkwise (WY / UT-transform) form of the gated delta rule
(Yang, Kautz, Hatamizadeh, "Gated Delta Networks", ICLR 2025), derived here from
the per-token recurrence H_i = g_i H_{i-1} + k_i beta_i (v_i - g_i H_{i-1}^T k_i).
Every exponent is Gamma_i - Gamma_j with j <= i, so no exp() overflows.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F


@torch.no_grad()
def prefill_chunked(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale=None, chunk=64,
                    dtype=torch.float64):
    T, HQ, D = q.shape
    HV = v.shape[1]
    N = cu_seqlens.numel() - 1
    if scale is None or float(scale) == 0.0:
        scale = 1.0 / math.sqrt(D)
    ratio = HV // HQ
    lg = (-torch.exp(A_log.to(dtype)) * F.softplus(a.to(dtype) + dt_bias.to(dtype)))  # [T,HV]
    beta = torch.sigmoid(b.to(dtype))
    qf = q.to(dtype).repeat_interleave(ratio, dim=1)
    kf = k.to(dtype).repeat_interleave(ratio, dim=1)
    vf = v.to(dtype)
    out = torch.zeros(T, HV, D, dtype=dtype)
    new_state = torch.zeros(N, HV, D, D, dtype=dtype)
    cu = [int(x) for x in cu_seqlens.tolist()]
    for n in range(N):
        s, e = cu[n], cu[n + 1]
        H = (state[n].to(dtype).transpose(-1, -2).clone() if state is not None
             else torch.zeros(HV, D, D, dtype=dtype))                       # [HV, K, V]
        for c0 in range(s, max(e, s), chunk):
            L = min(chunk, e - c0)
            idx = slice(c0, c0 + L)
            Kc = kf[idx].transpose(0, 1)                                  # [HV, L, K]
            Qc = qf[idx].transpose(0, 1)
            Vc = vf[idx].transpose(0, 1)
            G = torch.cumsum(lg[idx].transpose(0, 1), dim=-1)             # [HV, L]
            bt = beta[idx].transpose(0, 1)
            dG = G[:, :, None] - G[:, None, :]                            # Gamma_i - Gamma_j
            tril = torch.ones(L, L, dtype=torch.bool).tril()
            strict = tril & ~torch.eye(L, dtype=torch.bool)
            decay = torch.where(tril, torch.exp(torch.where(tril, dG, torch.zeros_like(dG))),
                                torch.zeros_like(dG))
            A = bt[:, :, None] * decay * (Kc @ Kc.transpose(-1, -2)) * strict
            M = decay * (Qc @ Kc.transpose(-1, -2))
            eye = torch.eye(L, dtype=dtype).expand(HV, L, L)
            Tb = torch.linalg.solve_triangular(eye + A, eye, upper=False) * bt[:, None, :]
            P = M @ Tb
            KH = Kc @ H
            QH = Qc @ H
            X = Vc - torch.exp(G)[:, :, None] * KH
            U = Tb @ X
            O = scale * (torch.exp(G)[:, :, None] * QH + P @ X)
            out[idx] = O.transpose(0, 1)
            Kt = torch.exp(G[:, -1:] - G)[:, :, None] * Kc
            H = torch.exp(G[:, -1])[:, None, None] * H + Kt.transpose(-1, -2) @ U
        new_state[n] = H.transpose(-1, -2)
    return out, new_state
