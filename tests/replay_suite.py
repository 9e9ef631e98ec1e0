"""A small workload suite in the flashinfer-bench record format (JSON lines plus a
safetensors file; the layout of the reference's scripts/setup_volume.py:32-140), written
to a directory for the replay tests."""
import json
import math
import uuid
from pathlib import Path

import torch
import torch.nn.functional as F


def write_suite(root: Path, seed: int = 0):
    from safetensors.torch import save_file
    g = torch.Generator().manual_seed(seed)
    scale = 1.0 / math.sqrt(128)
    (root / "workloads" / "gdn").mkdir(parents=True, exist_ok=True)
    tdir = root / "tensors" / "gdn_prefill"
    tdir.mkdir(parents=True, exist_ok=True)
    dec = []
    for bs in (1, 3):
        rnd = {n: {"type": "random"} for n in ("q", "k", "v", "state", "A_log", "a", "dt_bias", "b")}
        rnd["scale"] = {"type": "scalar", "value": scale}
        dec.append({"definition": "gdn_decode_qk4_v8_d128_k_last", "solution": None,
                    "workload": {"uuid": str(uuid.UUID(int=seed * 100 + bs)),
                                 "axes": {"batch_size": bs}, "inputs": rnd},
                    "evaluation": None})
    pre = []
    for total, n in ((130, 2), (64, 1)):
        wid = str(uuid.UUID(int=seed * 100 + 50 + total))
        seqlen = total // n
        cu = torch.tensor([min(i * seqlen, total) for i in range(n)] + [total], dtype=torch.int64)
        k = F.normalize(torch.randn(total, 4, 128, generator=g), dim=-1).to(torch.bfloat16)
        rel = f"tensors/gdn_prefill/tensors_{wid}.safetensors"
        save_file({"cu_seqlens": cu, "k": k, "state": torch.zeros(n, 8, 128, 128)},
                  str(root / rel))
        inputs = {n_: {"type": "random"} for n_ in ("q", "v", "A_log", "a", "dt_bias", "b")}
        inputs.update({"k": {"type": "safetensors", "path": rel, "tensor_key": "k"},
                       "state": {"type": "safetensors", "path": rel, "tensor_key": "state"},
                       "cu_seqlens": {"type": "safetensors", "path": rel,
                                      "tensor_key": "cu_seqlens"},
                       "scale": {"type": "scalar", "value": scale}})
        pre.append({"definition": "gdn_prefill_qk4_v8_d128_k_last", "solution": None,
                    "workload": {"uuid": wid, "axes": {"total_seq_len": total, "num_seqs": n,
                                                        "len_cu_seqlens": n + 1},
                                 "inputs": inputs},
                    "evaluation": None})
    (root / "workloads" / "gdn" / "gdn_decode.jsonl").write_text(
        "\n".join(json.dumps(r) for r in dec) + "\n")
    (root / "workloads" / "gdn" / "gdn_prefill.jsonl").write_text(
        "\n".join(json.dumps(r) for r in pre) + "\n")
    return root / "workloads" / "gdn"
