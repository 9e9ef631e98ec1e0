"""Workload replay (flashinfer_bench_tma_thrust_b200/replay.py): records of the official
suite's format materialise with the definition's shapes and dtypes (CPU), and replay
through the kernels matches the oracle (GPU)."""
import pytest
import torch

from flashinfer_bench_tma_thrust_b200 import replay
from oracle import gdn_oracle
from parity import DECODE_STATE_ATOL, PREFILL_STATE_ATOL, assert_out_close, assert_state_close
from replay_suite import write_suite


@pytest.fixture(scope="module")
def suite(tmp_path_factory):
    return write_suite(tmp_path_factory.mktemp("suite"))


def test_materialize_shapes_and_dtypes(suite):
    ws = list(replay.load_workloads(suite / "gdn_decode.jsonl"))
    assert [w.axes["batch_size"] for w in ws] == [1, 3]
    q, k, v, state, A_log, a, dt_bias, b, scale = ws[1].materialize("cpu")
    assert q.shape == (3, 1, 4, 128) and q.dtype == torch.bfloat16
    assert v.shape == (3, 1, 8, 128) and state.shape == (3, 8, 128, 128)
    assert state.dtype == torch.float32 and a.shape == (3, 1, 8) and a.dtype == torch.bfloat16
    assert A_log.shape == (8,) and abs(scale - 128 ** -0.5) < 1e-12
    again = ws[1].materialize("cpu")
    assert torch.equal(again[0], q)  # seeded by the uuid: a replay is repeatable
    ps = list(replay.load_workloads(suite / "gdn_prefill.jsonl"))
    q, k, v, state, A_log, a, dt_bias, b, cu, scale = ps[0].materialize("cpu")
    assert q.shape == (130, 4, 128) and v.shape == (130, 8, 128)
    assert cu.dtype == torch.int64 and cu.tolist() == [0, 65, 130]
    assert torch.equal(state, torch.zeros(2, 8, 128, 128))
    assert torch.allclose(k.float().norm(dim=-1), torch.ones(130, 4), atol=1e-2)
    out, ns = gdn_oracle.prefill(q, k, v, state, A_log, a, dt_bias, b, cu, scale)
    assert out.shape == (130, 8, 128) and torch.isfinite(out.float()).all()


def test_shape_mismatch_is_rejected(suite, tmp_path):
    ps = list(replay.load_workloads(suite / "gdn_prefill.jsonl"))
    w = ps[0]
    w.axes = dict(w.axes, total_seq_len=131)
    with pytest.raises(ValueError, match="shape"):
        w.materialize("cpu")


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["gdn_decode.jsonl", "gdn_prefill.jsonl"])
def test_replay_matches_oracle(suite, name):
    for w in replay.load_workloads(suite / name):
        args = w.materialize("cuda")
        out, ns = w.run(args)
        cpu = [t.cpu() if isinstance(t, torch.Tensor) else t for t in args]
        ref = gdn_oracle.decode(*cpu) if w.op == "decode" else gdn_oracle.prefill(*cpu)
        assert_out_close(out, ref[0], w.uuid)
        tol = DECODE_STATE_ATOL if w.op == "decode" else PREFILL_STATE_ATOL
        if w.op == "decode":  # unit-normal random state: absolute 1e-4 at unit scale
            err = (ns.cpu() - ref[1]).abs().max().item()
            assert err < 1e-4 * max(1.0, ref[1].abs().max().item()), (w.uuid, err)
        else:
            assert_state_close(ns, ref[1], tol, w.uuid)
        assert w.time_us(args, warmup=1, iters=3) > 0
