"""The chunk-64 algebra the CUDA prefill implements (oracle/gdn_chunked_model.py)
equals the reference's per-token recurrence (oracle/gdn_oracle.py, pinned to the
reference's golden outputs), including chunk boundaries, empty sequences and
strong-decay gates whose in-chunk cumulative log-decay reaches -1e3."""
import pytest
import torch

from flashinfer_bench_tma_thrust_b200 import workloads as W
from oracle import gdn_chunked_model, gdn_oracle


@pytest.mark.parametrize("lengths,dist", [
    ([1, 63, 64, 65, 0, 130], "baseline"),
    ([200], "reftest"),
    ([0, 7, 19, 3], "reftest"),
])
def test_chunk_form_equals_recurrence(lengths, dist):
    x = W.prefill_inputs(lengths, HQ=2, HV=4, seed=len(lengths), dist=dist)
    o_ref, s_ref = gdn_oracle.prefill(*x.args())
    o, s = gdn_chunked_model.prefill_chunked(*x.args())
    assert (o - o_ref.double()).abs().max().item() < 1e-2
    rel = ((s - s_ref.double()).norm() / s_ref.double().norm()).item()
    assert rel < 1e-5, rel


def test_chunk_form_no_overflow_under_strong_decay():
    x = W.prefill_inputs([128], HQ=1, HV=2, seed=3)
    x.a = x.a.float() + 30.0         # softplus ~ 30, exp(A_log) up to 16: log g ~ -480 per token
    o_ref, s_ref = gdn_oracle.prefill(*x.args())
    o, s = gdn_chunked_model.prefill_chunked(*x.args())
    assert torch.isfinite(o).all() and torch.isfinite(s).all()
    assert (o - o_ref.double()).abs().max().item() < 1e-2
    assert (s - s_ref.double()).abs().max().item() < 1e-5
