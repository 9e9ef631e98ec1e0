"""pytest configuration: the ``gpu`` marker and import paths.

``-m "not gpu"`` runs the oracle-vs-golden checks, host logic, the C-ABI
export check and the multi-process (gloo) partitioner tests on CPU.
``-m gpu`` runs the parity tests through the C ABI on a B200.
"""
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "tests"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU and the CUDA library")


@pytest.fixture(scope="session")
def cuda_lib():
    """The built C-ABI library (built here if missing; nvcc cross-compiles without a GPU)."""
    from flashinfer_bench_tma_thrust_b200 import _lib, build
    if not _lib.LIB_PATH.exists():
        build.build()
    return _lib.load()
