"""Stage the reference's own CPU implementation of the path for the bench's reference arm.

Test / measurement infrastructure, not product code. The reference's GDN baselines
(gdn/decode/baseline/triton/kernel.py and gdn/prefill/baseline/triton/kernel.py) are
pure PyTorch and run on the CPU unchanged; the checkout itself has no setup.py or
pyproject.toml, so it cannot be pip-installed. This copies those two files, as they
are, into baseline/_ref/ (git-ignored; it travels with the working tree to the GPU
box, where the checkout is absent), so that ``bench.py --impl reference`` and the
bench's ``cpu_baseline`` time the reference's own code ("kind": "reference"). Without
the staged files they fall back to the restatement in oracle/gdn_oracle.py ("port").
"""
from __future__ import annotations

import os
import shutil
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
FILES = ("gdn/decode/baseline/triton/kernel.py", "gdn/prefill/baseline/triton/kernel.py")


def stage(reference: str | os.PathLike | None = None) -> list[Path]:
    """Copy the baseline files from the reference checkout (``$GDN_REFERENCE_DIR``, by
    default the checkout mounted beside this repository) into baseline/_ref. Returns
    the staged paths; an empty list when the checkout is absent."""
    src_root = Path(reference or os.environ.get("GDN_REFERENCE_DIR", "/root/reference"))
    if not src_root.is_dir():
        return []
    out = []
    for rel in FILES:
        src = src_root / rel
        if not src.is_file():
            continue
        dst = ROOT / "baseline" / "_ref" / rel
        dst.parent.mkdir(parents=True, exist_ok=True)
        shutil.copyfile(src, dst)
        out.append(dst)
    return out


if __name__ == "__main__":
    for p in stage():
        print(p)
