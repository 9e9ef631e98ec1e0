"""Replay of flashinfer-bench workload records through the B200 GDN operators.

The official GDN suites (54 decode, 100 prefill workloads) are JSON-lines files of
workload records plus safetensors files (format of the reference's
scripts/setup_volume.py:32-140: per input a ``{"type": "random"}``, ``{"type":
"scalar", "value": v}`` or ``{"type": "safetensors", "path": p, "tensor_key": k}``
spec; variable axes in ``workload.axes``). The shapes and dtypes of each input come from
the operator definition (gdn/trace_definitions/*.json in the reference); this module
carries the two GDN definitions' axes, shapes and dtypes (the interface, restated) and
also reads a definition file given at run time (only its ``axes`` and ``inputs``).

``load_workloads(jsonl, root)`` yields ``Workload`` objects; ``Workload.materialize``
builds the argument tuple in the definition's order on a device (random inputs from a
generator seeded by the workload's uuid, so a replay is repeatable); ``run`` calls
``decode.kernel`` / ``prefill.kernel``; ``time_us`` times one workload with CUDA events.
Checking against a reference implementation is the caller's (the tests compare with
the CPU oracle).
"""
from __future__ import annotations

import hashlib
import json
from dataclasses import dataclass, field
from pathlib import Path

import torch

_DT = {"bfloat16": torch.bfloat16, "float32": torch.float32, "int64": torch.int64,
       "int32": torch.int32}


def _gdn_definition(op: str, hq: int, hv: int) -> dict:
    """Axes / inputs of the GDN decode or prefill definition at hq q/k heads and hv
    v-heads (the reference's gdn/trace_definitions/gdn_{op}_qk4_v8_d128_k_last.json at
    hq=4, hv=8)."""
    const = {"num_q_heads": hq, "num_k_heads": hq, "num_v_heads": hv, "head_size": 128}
    if op == "decode":
        const["seq_len"] = 1
        tok = ["batch_size", "seq_len"]
        state = ["batch_size", "num_v_heads", "head_size", "head_size"]
        inputs = {"q": tok + ["num_q_heads", "head_size"], "k": tok + ["num_k_heads", "head_size"],
                  "v": tok + ["num_v_heads", "head_size"], "state": state,
                  "A_log": ["num_v_heads"], "a": tok + ["num_v_heads"],
                  "dt_bias": ["num_v_heads"], "b": tok + ["num_v_heads"], "scale": None}
    else:
        tok = ["total_seq_len"]
        state = ["num_seqs", "num_v_heads", "head_size", "head_size"]
        inputs = {"q": tok + ["num_q_heads", "head_size"], "k": tok + ["num_k_heads", "head_size"],
                  "v": tok + ["num_v_heads", "head_size"], "state": state,
                  "A_log": ["num_v_heads"], "a": tok + ["num_v_heads"],
                  "dt_bias": ["num_v_heads"], "b": tok + ["num_v_heads"],
                  "cu_seqlens": ["len_cu_seqlens"], "scale": None}
    dtypes = {"q": "bfloat16", "k": "bfloat16", "v": "bfloat16", "state": "float32",
              "A_log": "float32", "a": "bfloat16", "dt_bias": "float32", "b": "bfloat16",
              "cu_seqlens": "int64", "scale": "float32"}
    return {"op": op,
            "axes": {k: {"type": "const", "value": v} for k, v in const.items()},
            "inputs": {k: {"shape": s, "dtype": dtypes[k]} for k, s in inputs.items()}}


DEFINITIONS = {
    "gdn_decode_qk4_v8_d128_k_last": _gdn_definition("decode", 4, 8),
    "gdn_prefill_qk4_v8_d128_k_last": _gdn_definition("prefill", 4, 8),
    "gdn_decode_qk16_v32_d128_k_last": _gdn_definition("decode", 16, 32),
    "gdn_prefill_qk16_v32_d128_k_last": _gdn_definition("prefill", 16, 32),
}


def load_definition(path) -> dict:
    """A definition file's axes and inputs (its embedded reference code is not used)."""
    d = json.loads(Path(path).read_text())
    op = "decode" if "decode" in d["name"] else "prefill"
    return {"op": op, "axes": d["axes"], "inputs": d["inputs"]}


@dataclass
class Workload:
    definition_name: str
    definition: dict
    uuid: str
    axes: dict
    inputs: dict
    root: Path
    extra: dict = field(default_factory=dict)

    @property
    def op(self) -> str:
        return self.definition["op"]

    def _axis(self, name: str) -> int:
        ax = self.definition["axes"].get(name, {"type": "var"})  # unlisted: variable
        if ax.get("type") == "const":
            return int(ax["value"])
        if name not in self.axes:
            raise KeyError(f"workload {self.uuid}: variable axis {name} has no value")
        return int(self.axes[name])

    def shape(self, name: str):
        spec = self.definition["inputs"][name]["shape"]
        return None if spec is None else tuple(self._axis(a) for a in spec)

    def materialize(self, device="cuda"):
        """Argument tuple in the definition's input order, on `device`."""
        seed = int(hashlib.sha256(self.uuid.encode()).hexdigest()[:8], 16)
        g = torch.Generator().manual_seed(seed)
        cache = {}
        args = []
        for name, idef in self.definition["inputs"].items():
            spec = self.inputs.get(name, {"type": "random"})
            dt = _DT[idef["dtype"]]
            kind = spec.get("type")
            if kind == "scalar":
                args.append(float(spec["value"]))
                continue
            if kind == "safetensors":
                from safetensors.torch import load_file
                path = self.root / spec["path"]
                if path not in cache:
                    cache[path] = load_file(str(path))
                t = cache[path][spec["tensor_key"]]
            elif kind == "random":
                shp = self.shape(name)
                if shp is None:  # a random scalar: the default scale
                    args.append(None)
                    continue
                if dt in (torch.int32, torch.int64):
                    raise ValueError(f"workload {self.uuid}: random integer input {name}")
                t = torch.randn(shp, generator=g)
            else:
                raise ValueError(f"workload {self.uuid}: input {name} of type {kind!r}")
            want = self.shape(name)
            if want is not None and tuple(t.shape) != want:
                raise ValueError(f"workload {self.uuid}: {name} has shape {tuple(t.shape)}, "
                                 f"the definition says {want}")
            args.append(t.to(dt).to(device))
        return tuple(args)

    def run(self, args):
        """(output, new_state) from the B200 operator."""
        if self.op == "decode":
            from . import decode
            return decode.kernel(*args)
        from . import prefill
        return prefill.kernel(*args)

    def time_us(self, args, warmup=3, iters=20) -> float:
        for _ in range(warmup):
            self.run(args)
        torch.cuda.synchronize()
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(iters):
            self.run(args)
        e.record()
        e.synchronize()
        return 1000.0 * s.elapsed_time(e) / iters


def load_workloads(jsonl, root=None, definitions=None):
    """Workload records of a JSON-lines file. `root` resolves safetensors paths (default:
    the directory of the file's parent suite, i.e. two levels up from the .jsonl as in
    the harness layout root/workloads/gdn/*.jsonl); `definitions` maps definition names
    to dicts of load_definition's form (default: the built-in GDN definitions)."""
    jsonl = Path(jsonl)
    root = Path(root) if root is not None else jsonl.parent.parent.parent
    defs = dict(DEFINITIONS)
    defs.update(definitions or {})
    for line in jsonl.read_text().splitlines():
        if not line.strip():
            continue
        rec = json.loads(line)
        name = rec["definition"]
        if name not in defs:
            raise KeyError(f"no definition for {name}")
        w = rec["workload"]
        yield Workload(name, defs[name], w["uuid"], w.get("axes", {}), w["inputs"], root,
                       {k: v for k, v in rec.items() if k not in ("definition", "workload")})
