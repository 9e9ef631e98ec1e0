"""Head ratios other than the configs' 2 (v-head h reads q/k head h // (HV/HQ), the
reference's repeat_interleave at gdn/decode/baseline/triton/kernel.py:69-71 and
gdn/prefill/baseline/triton/kernel.py:62): decode and every prefill implementation vs
the oracle at ratios 1, 4 and 8."""
import pytest

from flashinfer_bench_tma_thrust_b200 import decode, prefill, workloads as W
from oracle import gdn_oracle
from parity import (DECODE_STATE_ATOL, PREFILL_STATE_ATOL, assert_out_close,
                    assert_state_close, to_dev)

pytestmark = pytest.mark.gpu

RATIOS = [(4, 4), (2, 8), (1, 8), (1, 1)]
PREFILL = {"chunked": prefill.kernel, "fused": prefill.kernel_fused,
           "recurrent": prefill.kernel_recurrent}


@pytest.mark.parametrize("HQ,HV", RATIOS)
def test_decode_gva_ratio(HQ, HV):
    x = W.decode_inputs(5, HQ=HQ, HV=HV, seed=10 * HQ + HV)
    ref_out, ref_ns = gdn_oracle.decode(*x.args())
    out, ns = decode.kernel(*to_dev(x).args())
    assert out.shape == (5, 1, HV, 128) and ns.shape == (5, HV, 128, 128)
    assert_out_close(out, ref_out, f"decode HQ={HQ} HV={HV}")
    assert_state_close(ns, ref_ns, DECODE_STATE_ATOL, f"decode HQ={HQ} HV={HV}")


@pytest.mark.parametrize("impl", sorted(PREFILL))
@pytest.mark.parametrize("HQ,HV", RATIOS)
def test_prefill_gva_ratio(HQ, HV, impl):
    x = W.prefill_inputs([70, 0, 129], HQ=HQ, HV=HV, seed=10 * HQ + HV + 1)
    ref_out, ref_ns = gdn_oracle.prefill(*x.args())
    out, ns = PREFILL[impl](*to_dev(x).args())
    assert out.shape == (199, HV, 128) and ns.shape == (3, HV, 128, 128)
    assert_out_close(out, ref_out, f"{impl} HQ={HQ} HV={HV}")
    assert_state_close(ns, ref_ns, PREFILL_STATE_ATOL, f"{impl} HQ={HQ} HV={HV}")
