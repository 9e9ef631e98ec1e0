"""flashinfer-bench solution packaging (flashinfer_bench_tma_thrust_b200/solution.py):
the dict has the reference's structure (gdn/benchmarks/bench_modal.py:132-144), and
a materialised solution builds its library from the bundled sources and exposes
`kernel` through its entry file (compile only: no GPU needed)."""
import importlib.util
import json
import subprocess
import sys

import pytest

from flashinfer_bench_tma_thrust_b200 import solution


@pytest.mark.parametrize("op", ["decode", "prefill"])
def test_solution_dict_structure(op):
    d = solution.build_solution_dict(op)
    assert set(d) == {"name", "definition", "author", "spec", "sources"}
    assert d["spec"]["language"] == "cuda" and d["spec"]["entry_point"] == "kernel.py::kernel"
    assert d["spec"]["destination_passing_style"] is False
    paths = [s["path"] for s in d["sources"]]
    assert "kernel.py" in paths and "include/gdn_b200.h" in paths
    assert any(p.endswith("gdn_decode.cu") for p in paths)
    json.dumps(d)


def test_materialized_solution_builds_and_imports(tmp_path):
    d = solution.build_solution_dict("prefill")
    root = solution.materialize(d, tmp_path)
    code = ("import sys; sys.path.insert(0, %r); import kernel; "
            "print(kernel.kernel.__module__)" % str(root))
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=900,
                       cwd=str(root))
    assert r.returncode == 0, r.stderr[-2000:]
    assert "prefill" in r.stdout
    assert (root / "flashinfer_bench_tma_thrust_b200" / "libgdn_b200.so").exists()
