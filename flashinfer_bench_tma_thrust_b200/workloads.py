"""Seeded synthetic GDN workloads (stand-ins for the reference's official traces).

The reference's official 54 decode / 100 prefill workloads live in a dataset
that is not available here (scripts/setup_volume.py:180-200); its synthetic
generator only fixes shapes (scripts/setup_volume.py:32-140). These
generators produce the shapes and value distributions of the benchmark
configurations:

* ``dist="baseline"`` — q,k,v ~ N(0,1) drawn in fp32, q and k L2-normalised per
  head, then bf16; state ~ N(0, 0.02^2) fp32; A_log = log(U(1,16));
  dt_bias ~ U(-1,1); a, b ~ N(0,1) bf16.
* ``dist="reftest"`` — the distributions of the reference's prefill test
  (gdn/tests/test_correctness.py:474-482): q*0.1, L2-normalised k, v*0.1,
  state*0.01, A_log = 0.1 N - 1, a/b/dt_bias = 0.1 N, gates fp32.

Every tensor is drawn from one ``torch.Generator`` seeded with ``seed`` on
``gen_device`` and then moved to ``device``.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F

HQ_FULL, HV_FULL, D = 16, 32, 128


@dataclass
class DecodeInputs:
    q: torch.Tensor
    k: torch.Tensor
    v: torch.Tensor
    state: torch.Tensor | None
    A_log: torch.Tensor
    a: torch.Tensor
    dt_bias: torch.Tensor
    b: torch.Tensor
    scale: float

    def args(self):
        return (self.q, self.k, self.v, self.state, self.A_log, self.a, self.dt_bias, self.b,
                self.scale)


@dataclass
class PrefillInputs:
    q: torch.Tensor
    k: torch.Tensor
    v: torch.Tensor
    state: torch.Tensor | None
    A_log: torch.Tensor
    a: torch.Tensor
    dt_bias: torch.Tensor
    b: torch.Tensor
    cu_seqlens: torch.Tensor
    scale: float

    def args(self):
        return (self.q, self.k, self.v, self.state, self.A_log, self.a, self.dt_bias, self.b,
                self.cu_seqlens, self.scale)

    @property
    def lengths(self):
        cu = self.cu_seqlens.tolist()
        return [cu[i + 1] - cu[i] for i in range(len(cu) - 1)]


def _gen(seed: int, gen_device):
    g = torch.Generator(device=gen_device)
    g.manual_seed(seed)
    return g


def _qk(shape, g, gen_device, dist):
    x = torch.randn(*shape, generator=g, device=gen_device, dtype=torch.float32)
    if dist == "reftest":
        return x  # caller scales / normalises
    return F.normalize(x, dim=-1)


def _params(HV, lead, g, gen_device, dist, gate_dtype):
    if dist == "slowdecay":
        # the benchmark distributions with exp(A_log) ~ U(0.001, 0.05) instead of U(1, 16):
        # per-token decay g ~ 0.99, so the state survives many 64-token chunks (with the
        # benchmark's gates it decays to zero in fp32 within one chunk)
        A_log = torch.log(torch.rand(HV, generator=g, device=gen_device) * 0.049 + 0.001)
        dt_bias = torch.rand(HV, generator=g, device=gen_device) * 2.0 - 1.0
        a = torch.randn(*lead, HV, generator=g, device=gen_device)
        b = torch.randn(*lead, HV, generator=g, device=gen_device)
        gd = gate_dtype or torch.bfloat16
        return A_log.float(), a.to(gd), dt_bias.float(), b.to(gd)
    if dist == "baseline":
        A_log = torch.log(torch.rand(HV, generator=g, device=gen_device) * 15.0 + 1.0)
        dt_bias = torch.rand(HV, generator=g, device=gen_device) * 2.0 - 1.0
        a = torch.randn(*lead, HV, generator=g, device=gen_device)
        b = torch.randn(*lead, HV, generator=g, device=gen_device)
        gd = gate_dtype or torch.bfloat16
    else:
        A_log = torch.randn(HV, generator=g, device=gen_device) * 0.1 - 1.0
        a = torch.randn(*lead, HV, generator=g, device=gen_device) * 0.1
        dt_bias = torch.randn(HV, generator=g, device=gen_device) * 0.1
        b = torch.randn(*lead, HV, generator=g, device=gen_device) * 0.1
        gd = gate_dtype or torch.float32
    return A_log.float(), a.to(gd), dt_bias.float(), b.to(gd)


def decode_inputs(B, HQ=HQ_FULL, HV=HV_FULL, seed=0, device="cpu", gen_device="cpu",
                  dist="baseline", with_state=True, gate_dtype=None) -> DecodeInputs:
    g = _gen(seed, gen_device)
    if dist in ("baseline", "slowdecay"):
        q = _qk((B, 1, HQ, D), g, gen_device, dist)
        k = _qk((B, 1, HQ, D), g, gen_device, dist)
        v = torch.randn(B, 1, HV, D, generator=g, device=gen_device)
        state = torch.randn(B, HV, D, D, generator=g, device=gen_device) * 0.02 \
            if with_state else None
    else:
        q = _qk((B, 1, HQ, D), g, gen_device, dist) * 0.1
        k = F.normalize(_qk((B, 1, HQ, D), g, gen_device, dist), dim=-1)
        v = torch.randn(B, 1, HV, D, generator=g, device=gen_device) * 0.1
        state = torch.randn(B, HV, D, D, generator=g, device=gen_device) * 0.01 \
            if with_state else None
    A_log, a, dt_bias, b = _params(HV, (B, 1), g, gen_device, dist, gate_dtype)
    t = lambda x: None if x is None else x.to(device)  # noqa: E731
    return DecodeInputs(t(q.to(torch.bfloat16)), t(k.to(torch.bfloat16)),
                        t(v.to(torch.bfloat16)), t(state), t(A_log), t(a), t(dt_bias), t(b),
                        1.0 / math.sqrt(D))


def prefill_inputs(lengths, HQ=HQ_FULL, HV=HV_FULL, seed=0, device="cpu", gen_device="cpu",
                   dist="baseline", with_state=True, cu_dtype=torch.int32,
                   gate_dtype=None) -> PrefillInputs:
    g = _gen(seed, gen_device)
    T = int(sum(lengths))
    N = len(lengths)
    if dist in ("baseline", "slowdecay"):
        q = _qk((T, HQ, D), g, gen_device, dist)
        k = _qk((T, HQ, D), g, gen_device, dist)
        v = torch.randn(T, HV, D, generator=g, device=gen_device)
        state = torch.randn(N, HV, D, D, generator=g, device=gen_device) * 0.02 \
            if with_state else None
    else:
        q = _qk((T, HQ, D), g, gen_device, dist) * 0.1
        k = F.normalize(_qk((T, HQ, D), g, gen_device, dist), dim=-1)
        v = torch.randn(T, HV, D, generator=g, device=gen_device) * 0.1
        state = torch.randn(N, HV, D, D, generator=g, device=gen_device) * 0.01 \
            if with_state else None
    A_log, a, dt_bias, b = _params(HV, (T,), g, gen_device, dist, gate_dtype)
    cu = torch.zeros(N + 1, dtype=torch.int64)
    if N:
        cu[1:] = torch.cumsum(torch.tensor(lengths, dtype=torch.int64), 0)
    t = lambda x: None if x is None else x.to(device)  # noqa: E731
    return PrefillInputs(t(q.to(torch.bfloat16)), t(k.to(torch.bfloat16)),
                         t(v.to(torch.bfloat16)), t(state), t(A_log), t(a), t(dt_bias), t(b),
                         cu.to(cu_dtype).to(device), 1.0 / math.sqrt(D))


def varlen_lengths(seed=0, n=8, lo=512, hi=4096):
    """Config 4: 8 lengths ~ U[512, 4096] from a seeded generator."""
    g = torch.Generator().manual_seed(seed)
    return torch.randint(lo, hi + 1, (n,), generator=g).tolist()
