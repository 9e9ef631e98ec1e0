"""Loader for ``gdn_golden.npz`` (written by ``make_golden.py`` from the reference).

``load_case(name)`` returns ``(kind, inputs, expected)``: ``inputs`` is a
``workloads.DecodeInputs`` / ``PrefillInputs`` on the CPU, ``expected`` a dict
with ``out`` (bf16) and either ``new_state`` (fp32) or the digest arrays
``new_state.rowsum`` / ``.rowsq`` / ``.rows16``. Inputs that were stored only as a
hash are regenerated from the stored seed and checked against that hash.
"""
from __future__ import annotations

import hashlib
import json
from functools import lru_cache
from pathlib import Path

import numpy as np
import torch

from flashinfer_bench_tma_thrust_b200 import workloads as W

PATH = Path(__file__).resolve().parent / "gdn_golden.npz"
INPUT_NAMES = ("q", "k", "v", "state", "A_log", "a", "dt_bias", "b", "cu_seqlens")


@lru_cache(maxsize=1)
def _npz():
    z = np.load(PATH)
    return {k: z[k] for k in z.files}


def case_names():
    return sorted({k.split("/")[0] for k in _npz()})


def _torch(arr: np.ndarray, dtype: str) -> torch.Tensor:
    if dtype == "bfloat16":
        return torch.from_numpy(arr.view(np.int16).copy()).view(torch.bfloat16)
    return torch.from_numpy(arr.copy())


def _sha(t: torch.Tensor) -> str:
    t = t.contiguous()
    a = t.view(torch.int16).numpy().view(np.uint16) if t.dtype == torch.bfloat16 else t.numpy()
    return hashlib.sha256(a.tobytes()).hexdigest()


def state_digest(s: torch.Tensor) -> dict:
    s = s.float()
    return {"rowsum": s.sum(-1), "rowsq": (s * s).sum(-1), "rows16": s[:, :, ::16, :]}


def load_case(name: str):
    z = _npz()
    pre = f"{name}/"
    params = json.loads(str(z[pre + "params"])) if pre + "params" in z else None
    regen = None
    if params is not None and any(pre + f"{n}.sha256" in z for n in INPUT_NAMES):
        if params["kind"] == "decode":
            gd = getattr(torch, params["gate_dtype"]) if params["gate_dtype"] else None
            regen = W.decode_inputs(params["B"], params["HQ"], params["HV"], seed=params["seed"],
                                    dist=params["dist"], with_state=params["with_state"],
                                    gate_dtype=gd)
        else:
            regen = W.prefill_inputs(params["lengths"], params["HQ"], params["HV"],
                                     seed=params["seed"], dist=params["dist"],
                                     with_state=params["with_state"],
                                     cu_dtype=getattr(torch, params["cu_dtype"]))
    vals = {}
    for n in INPUT_NAMES:
        if pre + n in z:
            vals[n] = _torch(z[pre + n], str(z[pre + n + ".dtype"]))
        elif pre + n + ".sha256" in z:
            t = getattr(regen, n)
            if _sha(t) != str(z[pre + n + ".sha256"]):
                raise RuntimeError(f"golden case {name}: regenerated input {n} does not match "
                                   "its stored hash (generator drift)")
            vals[n] = t
        else:
            vals[n] = None
    scale = float(z[pre + "scale"])
    kind = "prefill" if vals["cu_seqlens"] is not None else "decode"
    if kind == "decode":
        inputs = W.DecodeInputs(vals["q"], vals["k"], vals["v"], vals["state"], vals["A_log"],
                                vals["a"], vals["dt_bias"], vals["b"], scale)
    else:
        inputs = W.PrefillInputs(vals["q"], vals["k"], vals["v"], vals["state"], vals["A_log"],
                                 vals["a"], vals["dt_bias"], vals["b"], vals["cu_seqlens"], scale)
    expected = {"out": _torch(z[pre + "out"], str(z[pre + "out.dtype"]))}
    if pre + "new_state" in z:
        expected["new_state"] = _torch(z[pre + "new_state"], "float32")
    else:
        for d in ("rowsum", "rowsq", "rows16"):
            expected[f"new_state.{d}"] = torch.from_numpy(z[pre + f"new_state.{d}"].copy())
    return kind, inputs, expected


def compare_state(new_state: torch.Tensor, expected: dict, atol: float, rtol_frob: float):
    """Return (max_abs_err, rel_frobenius_err) of new_state against the golden record
    (full tensor when stored, else the digest rows plus row sums)."""
    ns = new_state.detach().float().cpu()
    if "new_state" in expected:
        ref = expected["new_state"]
        got = ns
    else:
        d = state_digest(ns)
        ref = expected["new_state.rows16"]
        got = d["rows16"]
        rs = (d["rowsum"] - expected["new_state.rowsum"]).abs().max().item()
        rq = ((d["rowsq"] - expected["new_state.rowsq"]).abs() /
              expected["new_state.rowsq"].abs().clamp_min(1e-12)).max().item()
        if rs > atol * 128 or rq > 10 * rtol_frob:
            return float("inf"), float("inf")
    err = (got - ref).abs().max().item()
    rel = ((got - ref).norm() / ref.norm().clamp_min(1e-30)).item()
    return err, rel
