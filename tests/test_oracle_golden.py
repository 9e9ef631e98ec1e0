"""Pin the CPU oracle (oracle/gdn_oracle.py) to the reference's own outputs.

Every case in tests/golden/gdn_golden.npz was produced by running the
reference's PyTorch baselines (gdn/decode/baseline/triton/kernel.py,
gdn/prefill/baseline/triton/kernel.py) on the stored inputs. The oracle must
reproduce them to fp32 round-off: out within one bf16 ulp, state within 1e-5.
"""
import pytest
import torch

from golden import golden
from oracle import gdn_oracle

CASES = golden.case_names()


@pytest.mark.parametrize("name", CASES)
def test_oracle_matches_reference_golden(name):
    kind, x, exp = golden.load_case(name)
    fn = gdn_oracle.decode if kind == "decode" else gdn_oracle.prefill
    out, ns = fn(*x.args())
    ref_out = exp["out"].float()
    # one bf16 ulp at the output magnitude
    tol = ref_out.abs().clamp_min(1e-3) * 2.0 ** -7 + 1e-6
    assert ((out.float() - ref_out).abs() <= tol).all(), name
    err, rel = golden.compare_state(ns, exp, atol=1e-5, rtol_frob=1e-6)
    assert err < 1e-5 and rel < 1e-6, (name, err, rel)


def test_known_answer_gates():
    """A_log=a=dt_bias=b=0 gives g = exp(-ln 2) = 0.5 and beta = 0.5
    (gdn/tests/test_correctness.py:323-336, printed there, asserted here)."""
    z = torch.zeros(4)
    g, beta = gdn_oracle.gates(z, z, z, z)
    assert torch.allclose(g, torch.full((4,), 0.5), atol=1e-7)
    assert torch.allclose(beta, torch.full((4,), 0.5), atol=1e-7)


def test_known_answer_decode_closed_form():
    """Uniform inputs: state ones, q=k=v=0.1 (bf16), g=beta=0.5. Every row of the
    new state is 0.5*1 + 0.5*(0.1 - 0.5*sum(k))*k, fully determined."""
    kind, x, exp = golden.load_case("dec_known_answer")
    out, ns = gdn_oracle.decode(*x.args())
    kv = x.k.float()[0, 0, 0]
    old = 0.5 * kv.sum()
    delta = 0.5 * (x.v.float()[0, 0, 0, 0] - old)
    row = 0.5 + delta * kv
    assert torch.allclose(ns[0, 0, 0], row, atol=1e-6)
    o = x.scale * (row * x.q.float()[0, 0, 0]).sum()
    assert abs(out.float()[0, 0, 0, 0].item() - o.item()) < 1e-2
