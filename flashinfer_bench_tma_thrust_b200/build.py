"""Build the sm_100a shared library ``libgdn_b200.so`` in-tree with nvcc.

The library is the C-ABI boundary declared in ``include/gdn_b200.h``. It is
compiled directly with nvcc (no torch extension machinery), so the same ``.so``
can be bound from ctypes, cffi or any other FFI. Built objects are cached under
``flashinfer_bench_tma_thrust_b200/_build`` and relinked only when a source changed.
"""
from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
INCLUDE = REPO_DIR / "include"
BUILD_DIR = PKG_DIR / "_build"
LIB_PATH = PKG_DIR / "libgdn_b200.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    # full-precision math: gates use expf/log1pf and must match the fp32 reference
]

SOURCES = sorted(CSRC.glob("*.cu"))
HEADERS = sorted(list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h")))


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: cannot build the GDN CUDA library")
    return cand


def _digest(paths, extra: str = "") -> str:
    h = hashlib.sha256(extra.encode())
    for p in paths:
        h.update(p.name.encode())
        h.update(p.read_bytes())
    return h.hexdigest()[:16]


def build(verbose: bool = False, force: bool = False, ptxas_verbose: bool = False) -> Path:
    """Compile every ``csrc/*.cu`` for sm_100a and link ``libgdn_b200.so``."""
    nvcc = _nvcc()
    BUILD_DIR.mkdir(exist_ok=True)
    header_digest = _digest(HEADERS, " ".join(ARCH_FLAGS + NVCC_FLAGS))
    objs = []
    for src in SOURCES:
        key = _digest([src], header_digest)
        obj = BUILD_DIR / f"{src.stem}.{key}.o"
        objs.append(obj)
        if obj.exists() and not force:
            continue
        for stale in BUILD_DIR.glob(f"{src.stem}.*.o"):
            stale.unlink()
        cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, f"-I{INCLUDE}", f"-I{CSRC}", "-c", str(src),
               "-o", str(obj)]
        if ptxas_verbose:
            cmd[1:1] = ["-Xptxas", "-v"]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
    link_key = _digest(objs)
    stamp = BUILD_DIR / "link.stamp"
    if LIB_PATH.exists() and stamp.exists() and stamp.read_text() == link_key and not force:
        return LIB_PATH
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs), "-lcuda"]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB_PATH)
    stamp.write_text(link_key)
    return LIB_PATH


if __name__ == "__main__":
    import argparse

    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas", action="store_true", help="print ptxas register/smem usage")
    args = ap.parse_args()
    print(build(verbose=args.verbose, force=args.force, ptxas_verbose=args.ptxas))
