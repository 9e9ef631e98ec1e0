"""Build recipe for oracle/_ref/: the reference's own GPU decode kernel as a bench-only
comparator (measurement infrastructure, not the product; nothing in the package links
or imports it).

    python oracle/build_ref.py            # -> oracle/_ref/libref_v10.so

Compiles oracle/ref_v10_decode.cu (a C entry point of this repository) against the
reference's header gdn/kernels/cute_cpp/gdn_decode_v10.cuh, read where it lies in the
reference checkout ($GDN_REFERENCE_DIR, default the checkout mounted beside this
repository), with the CuTe headers that ship inside the installed flashinfer package.
Nothing is copied. Without the checkout or the headers it builds nothing; the bench then
reports the comparator as unavailable.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref" / "libref_v10.so"


def _cute_include():
    try:
        import flashinfer
    except Exception:  # noqa: BLE001 - the comparator is optional
        return None
    p = Path(flashinfer.__file__).resolve().parent / "data" / "cutlass" / "include"
    return p if (p / "cute").is_dir() else None


def build(force: bool = False):
    ref = Path(os.environ.get("GDN_REFERENCE_DIR", "/root/reference"))
    hdr_dir = ref / "gdn" / "kernels" / "cute_cpp"
    cute = _cute_include()
    if not (hdr_dir / "gdn_decode_v10.cuh").is_file() or cute is None:
        return None
    src = HERE / "ref_v10_decode.cu"
    if OUT.exists() and not force and OUT.stat().st_mtime > src.stat().st_mtime:
        return OUT
    OUT.parent.mkdir(exist_ok=True)
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17",
           "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC", "-shared",
           f"-I{hdr_dir}", f"-I{cute}", str(src), "-o", str(OUT)]
    subprocess.run(cmd, check=True)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
