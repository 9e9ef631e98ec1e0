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


_RUN_PACKAGED = r"""
import sys, torch
sys.path.insert(0, sys.argv[1])
import kernel
inp = torch.load(sys.argv[2])
args = [t.cuda() if isinstance(t, torch.Tensor) else t for t in inp]
out, ns = kernel.kernel(*args)
torch.cuda.synchronize()
torch.save((out.cpu(), ns.cpu(), kernel.kernel.__module__), sys.argv[3])
"""


@pytest.mark.gpu
@pytest.mark.parametrize("op", ["decode", "prefill"])
def test_materialized_solution_kernel_matches_oracle(op, tmp_path):
    """The packaged solution as a harness would run it: materialise the dict, import its
    generated kernel.py::kernel in a fresh process (which builds the library from the
    bundled sources), call it on the GPU and compare with the CPU oracle."""
    import torch
    from flashinfer_bench_tma_thrust_b200 import workloads as W
    from oracle import gdn_oracle
    from parity import (DECODE_STATE_ATOL, PREFILL_STATE_ATOL, assert_out_close,
                        assert_state_close)
    root = solution.materialize(solution.build_solution_dict(op), tmp_path / "sol")
    if op == "decode":
        x = W.decode_inputs(8, seed=12)
        ref = gdn_oracle.decode(*x.args())
        atol = DECODE_STATE_ATOL
    else:
        x = W.prefill_inputs([130, 0, 64, 7], seed=13)
        ref = gdn_oracle.prefill(*x.args())
        atol = PREFILL_STATE_ATOL
    torch.save(list(x.args()), tmp_path / "in.pt")
    script = tmp_path / "run.py"
    script.write_text(_RUN_PACKAGED)
    r = subprocess.run([sys.executable, str(script), str(root), str(tmp_path / "in.pt"),
                        str(tmp_path / "res.pt")], capture_output=True, text=True,
                       timeout=900, cwd=str(root))
    assert r.returncode == 0, r.stderr[-2000:]
    out, ns, module = torch.load(tmp_path / "res.pt")
    assert module.endswith(op)
    assert_out_close(out, ref[0], f"packaged {op}")
    assert_state_close(ns, ref[1], atol, f"packaged {op}")
