"""Generate the golden GDN fixtures by running the REFERENCE's own PyTorch code.

Run once, in a checkout where the reference repository is available:

    python tests/golden/make_golden.py --reference <path-to-reference-checkout>

It imports the reference's baseline kernels by file path
(gdn/decode/baseline/triton/kernel.py, gdn/prefill/baseline/triton/kernel.py —
pure PyTorch despite the directory name, no head-count asserts), runs them on
the CPU on seeded inputs and writes ``gdn_golden.npz`` next to this script.
The fixtures carry inputs and outputs, so the tests that read them never need
the reference. bf16 tensors are stored as their raw uint16 bits.

Cases cover what the reference's tests cover (gdn/tests/test_correctness.py):
decode batches with and without state and with fp32 gates (:193-224), the
gate known answer A_log=a=dt_bias=b=0 => g=0.5, beta=0.5 (:323-336), and
prefill lengths [32], [0,7,19,3], [1,2,4,8,0,5] with empty sequences and int32
cu_seqlens (:450-488); plus int64 cu_seqlens, a no-state prefill, a
multi-chunk sequence (lengths crossing 64-token chunk boundaries) and one
full-head (16 q/k, 32 v) decode and prefill at the benchmark distributions.
Head counts are kept small in most cases to keep the file small.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import importlib.util
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from flashinfer_bench_tma_thrust_b200 import workloads as W  # noqa: E402


def _load(path: Path, name: str):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _np(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


FULL_LIMIT = 140_000  # bytes; larger inputs are stored as a hash (and regenerated
#                       from the stored seed), a larger new_state as a digest


def _sha(t: torch.Tensor) -> str:
    return hashlib.sha256(_np(t).tobytes()).hexdigest()


def state_digest(s: torch.Tensor) -> dict:
    """Size-reduced fingerprint of a [N,HV,V,K] fp32 state: per-row sums and sums of
    squares plus every 16th row in full (the tests compare these within tolerance)."""
    s = s.float()
    return {"rowsum": s.sum(-1), "rowsq": (s * s).sum(-1), "rows16": s[:, :, ::16, :].contiguous()}


def _put(store: dict, case: str, **tensors):
    for k, v in tensors.items():
        if v is None:
            continue
        if isinstance(v, torch.Tensor) and k not in ("out",) and \
                v.numel() * v.element_size() > FULL_LIMIT:
            if k != "new_state":
                store[f"{case}/{k}.sha256"] = np.array(_sha(v))
            else:
                for dk, dv in state_digest(v).items():
                    store[f"{case}/new_state.{dk}"] = _np(dv)
            continue
        if isinstance(v, torch.Tensor):
            store[f"{case}/{k}"] = _np(v)
            store[f"{case}/{k}.dtype"] = np.array(str(v.dtype).replace("torch.", ""))
        else:
            store[f"{case}/{k}"] = np.array(v)


DECODE_CASES = [
    # name, B, HQ, HV, dist, with_state, gate_dtype, seed
    ("dec_b1_h1x2", 1, 1, 2, "baseline", True, None, 42),
    ("dec_b3_h2x4", 3, 2, 4, "baseline", True, None, 43),
    ("dec_b2_reftest_f32gates", 2, 1, 2, "reftest", True, torch.float32, 44),
    ("dec_b2_nostate", 2, 1, 2, "baseline", False, None, 45),
    ("dec_b1_full16x32", 1, 16, 32, "baseline", True, None, 46),
]

PREFILL_CASES = [
    # name, lengths, HQ, HV, dist, with_state, cu_dtype, seed
    ("pre_single32", [32], 1, 2, "reftest", True, torch.int32, 1234 + 32 + 1),
    ("pre_varlen_empty", [0, 7, 19, 3], 1, 2, "reftest", True, torch.int32, 1234 + 29 + 4),
    ("pre_mixed_short", [1, 2, 4, 8, 0, 5], 1, 2, "reftest", True, torch.int64, 1234 + 20 + 6),
    ("pre_nostate", [5, 17, 0, 9], 1, 2, "baseline", False, torch.int64, 7),
    ("pre_multichunk", [130, 64, 63, 65], 1, 2, "baseline", True, torch.int32, 8),
    ("pre_multichunk_reftest", [200], 2, 4, "reftest", True, torch.int32, 9),
    ("pre_full16x32", [66, 0, 5], 16, 32, "baseline", True, torch.int32, 10),
]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference checkout")
    ap.add_argument("--out", default=str(HERE / "gdn_golden.npz"))
    args = ap.parse_args()
    ref = Path(args.reference)
    dec = _load(ref / "gdn/decode/baseline/triton/kernel.py", "ref_gdn_decode_baseline")
    pre = _load(ref / "gdn/prefill/baseline/triton/kernel.py", "ref_gdn_prefill_baseline")
    torch.set_num_threads(max(1, torch.get_num_threads()))
    store: dict = {}
    for name, B, HQ, HV, dist, ws, gd, seed in DECODE_CASES:
        x = W.decode_inputs(B, HQ, HV, seed=seed, dist=dist, with_state=ws, gate_dtype=gd)
        out, ns = dec.kernel(*x.args())
        store[f"{name}/params"] = np.array(json.dumps(dict(
            kind="decode", B=B, HQ=HQ, HV=HV, dist=dist, with_state=ws, seed=seed,
            gate_dtype=None if gd is None else str(gd).replace("torch.", ""))))
        _put(store, name, q=x.q, k=x.k, v=x.v, state=x.state, A_log=x.A_log, a=x.a,
             dt_bias=x.dt_bias, b=x.b, scale=x.scale, out=out, new_state=ns.contiguous())
    # gate known answer (gdn/tests/test_correctness.py:323-336): g = 0.5, beta = 0.5
    B, HQ, HV, D = 1, 1, 2, 128
    q = torch.full((B, 1, HQ, D), 0.1).to(torch.bfloat16)
    k = q.clone()
    v = torch.full((B, 1, HV, D), 0.1).to(torch.bfloat16)
    st = torch.ones(B, HV, D, D)
    z = torch.zeros(HV)
    zab = torch.zeros(B, 1, HV)
    out, ns = dec.kernel(q, k, v, st, z, zab, z, zab, 1.0 / np.sqrt(D))
    _put(store, "dec_known_answer", q=q, k=k, v=v, state=st, A_log=z, a=zab, dt_bias=z, b=zab,
         scale=float(1.0 / np.sqrt(D)), out=out, new_state=ns.contiguous())
    for name, lengths, HQ, HV, dist, ws, cd, seed in PREFILL_CASES:
        x = W.prefill_inputs(lengths, HQ, HV, seed=seed, dist=dist, with_state=ws, cu_dtype=cd)
        out, ns = pre.kernel(*x.args())
        store[f"{name}/params"] = np.array(json.dumps(dict(
            kind="prefill", lengths=lengths, HQ=HQ, HV=HV, dist=dist, with_state=ws, seed=seed,
            cu_dtype=str(cd).replace("torch.", ""))))
        _put(store, name, q=x.q, k=x.k, v=x.v, state=x.state, A_log=x.A_log, a=x.a,
             dt_bias=x.dt_bias, b=x.b, cu_seqlens=x.cu_seqlens, scale=x.scale, out=out,
             new_state=ns.contiguous())
    np.savez_compressed(args.out, **store)
    size = Path(args.out).stat().st_size
    print(f"wrote {args.out} ({size / 1e6:.2f} MB, {len(store)} arrays)")


if __name__ == "__main__":
    main()
