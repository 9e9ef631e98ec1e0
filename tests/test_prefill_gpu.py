"""Prefill parity on the GPU: chunked (kernel) and token-sequential (kernel_recurrent)
sm_100a kernels through the C ABI vs the oracle and the reference's golden outputs."""
import pytest
import torch

from flashinfer_bench_tma_thrust_b200 import prefill, workloads as W
from golden import golden
from oracle import gdn_oracle
from parity import (PREFILL_STATE_ATOL, STATE_REL_FROB, assert_out_close, assert_state_close,
                    to_dev)

pytestmark = pytest.mark.gpu

PRE_CASES = [c for c in golden.case_names() if c.startswith("pre_")]
IMPLS = {"chunked": prefill.kernel, "fused": prefill.kernel_fused,
         "recurrent": prefill.kernel_recurrent}


@pytest.mark.parametrize("impl", sorted(IMPLS))
@pytest.mark.parametrize("name", PRE_CASES)
def test_prefill_matches_reference_golden(name, impl):
    _, x, exp = golden.load_case(name)
    out, ns = IMPLS[impl](*to_dev(x).args())
    assert_out_close(out, exp["out"], name)
    err, rel = golden.compare_state(ns, exp, atol=PREFILL_STATE_ATOL, rtol_frob=STATE_REL_FROB)
    assert err <= PREFILL_STATE_ATOL and rel <= STATE_REL_FROB, (name, err, rel)


LENGTHS = [
    [1], [63], [64], [65], [128], [200, 0, 1, 64, 127],
    [0, 0], [300, 17],
    [129, 192, 193, 256],  # 3-4 chunks: the pipelined scan's prologue, steady state, tail
]


@pytest.mark.parametrize("impl", sorted(IMPLS))
@pytest.mark.parametrize("lengths", LENGTHS, ids=lambda l: "-".join(map(str, l)))
def test_prefill_full_heads_vs_oracle(lengths, impl):
    x = W.prefill_inputs(lengths, seed=sum(lengths) + len(lengths))
    ref_out, ref_ns = gdn_oracle.prefill(*x.args())
    out, ns = IMPLS[impl](*to_dev(x).args())
    assert out.shape == (sum(lengths), 32, 128) and ns.shape == (len(lengths), 32, 128, 128)
    assert_out_close(out, ref_out, str(lengths))
    assert_state_close(ns, ref_ns, PREFILL_STATE_ATOL, str(lengths))


@pytest.mark.parametrize("impl", sorted(IMPLS))
@pytest.mark.parametrize("dist", ["baseline", "reftest"])
def test_prefill_no_state_int64_bf16_gates(impl, dist):
    x = W.prefill_inputs([70, 5, 0, 130], HQ=4, HV=8, seed=3, dist=dist, with_state=False,
                         cu_dtype=torch.int64, gate_dtype=torch.bfloat16)
    ref_out, ref_ns = gdn_oracle.prefill(*x.args())
    out, ns = IMPLS[impl](*to_dev(x).args())
    assert_out_close(out, ref_out)
    assert_state_close(ns, ref_ns, PREFILL_STATE_ATOL)
    assert torch.count_nonzero(ns[2]) == 0  # empty sequence, no initial state -> zeros


@pytest.mark.parametrize("impl", sorted(IMPLS))
def test_prefill_empty_sequence_passthrough_exact(impl):
    """Empty sequences copy their state through (reference threshold < 1e-6,
    gdn/tests/test_correctness.py:506-514); here it must be bit-exact."""
    x = to_dev(W.prefill_inputs([0, 9, 0], HQ=2, HV=4, seed=5))
    s0 = x.state.clone()
    out, ns = IMPLS[impl](*x.args())
    assert torch.equal(ns[0], s0[0]) and torch.equal(ns[2], s0[2])
    assert torch.equal(x.state, s0), "inputs must not be modified"


@pytest.mark.parametrize("impl", sorted(IMPLS))
def test_prefill_all_empty(impl):
    x = to_dev(W.prefill_inputs([0, 0, 0], HQ=2, HV=4, seed=6))
    out, ns = IMPLS[impl](*x.args())
    assert out.shape == (0, 4, 128)
    assert torch.equal(ns, x.state)


def test_chunked_vs_recurrent_varlen_config():
    """Config 4 shapes (8 sequences, lengths ~U[512,4096], 32 v-heads): the two independent
    CUDA implementations agree, at a size where the CPU oracle would take minutes."""
    lengths = W.varlen_lengths(seed=0)
    x = W.prefill_inputs(lengths, seed=21, gen_device="cuda", device="cuda")
    o1, s1 = prefill.kernel(*x.args())
    o2, s2 = prefill.kernel_recurrent(*x.args())
    o3, s3 = prefill.kernel_fused(*x.args())
    assert_out_close(o1, o2, "chunked vs recurrent")
    assert_state_close(s1, s2, PREFILL_STATE_ATOL, "chunked vs recurrent")
    assert_out_close(o3, o2, "fused vs recurrent")
    assert_state_close(s3, s2, PREFILL_STATE_ATOL, "fused vs recurrent")


def test_chunked_vs_recurrent_long_sequence():
    """Config 5's sequence length (32,768 tokens = 512 chunks) plus a ragged second
    sequence: the chunk-64 path stays within the parity tolerances of the token-by-token
    fp32 recurrence over the whole length (a size-independent check at full size)."""
    x = W.prefill_inputs([32768, 1000], seed=77, gen_device="cuda", device="cuda")
    o1, s1 = prefill.kernel(*x.args())
    o2, s2 = prefill.kernel_recurrent(*x.args())
    assert_out_close(o1, o2, "chunked vs recurrent, 32768 tokens")
    assert_state_close(s1, s2, PREFILL_STATE_ATOL, "chunked vs recurrent, 32768 tokens")


@pytest.mark.parametrize("n_seqs", [1024, 1100])
def test_chunked_many_sequences(n_seqs):
    """Many short ragged sequences (empty ones included) on both sides of the 1024-sequence
    limit up to which the chunk-offsets kernel also computes the scan order (above it a
    separate launch does): the chunked path agrees with the token-sequential kernel."""
    g = torch.Generator().manual_seed(n_seqs)
    lengths = torch.randint(0, 80, (n_seqs,), generator=g).tolist()
    x = W.prefill_inputs(lengths, seed=5, gen_device="cuda", device="cuda")
    o1, s1 = prefill.kernel(*x.args())
    o2, s2 = prefill.kernel_recurrent(*x.args())
    assert_out_close(o1, o2, f"chunked vs recurrent, {n_seqs} sequences")
    assert_state_close(s1, s2, PREFILL_STATE_ATOL, f"chunked vs recurrent, {n_seqs} sequences")
    torch.cuda.synchronize()
    assert prefill.device_status() == 0


def test_split_call_matches_unsplit(monkeypatch):
    """Few long sequences (4 x 8192 tokens, 32 v-heads: 128 scan chains, SMs left idle):
    the call is split (the prep of each sequence's last chunks overlaps the first part
    of the scan) and must agree with the unsplit call (GDN_PREFILL_OVERLAP=0): the state
    chain is the same fp32 arithmetic; the output of the first chunk after the split
    takes its state product in one piece instead of two."""
    x = W.prefill_inputs([8192] * 4, seed=13, gen_device="cuda", device="cuda")
    monkeypatch.setenv("GDN_PREFILL_OVERLAP", "0")
    o1, s1 = prefill.kernel(*x.args())
    monkeypatch.setenv("GDN_PREFILL_OVERLAP", "1")
    o2, s2 = prefill.kernel(*x.args())
    torch.cuda.synchronize()
    assert_out_close(o2, o1, "split vs unsplit")
    assert_state_close(s2, s1, PREFILL_STATE_ATOL, "split vs unsplit")
    assert prefill.device_status() == 0


def test_chunked_status_word_clean():
    """Every bounded wait inside the chunked kernel completed in the calls above."""
    x = to_dev(W.prefill_inputs([130, 7], HQ=2, HV=4, seed=31))
    prefill.kernel(*x.args())
    torch.cuda.synchronize()
    assert prefill.device_status() == 0


def test_partitioned_prefill_reassembles_to_full_call():
    """A 4-rank plan (heads split: 3 sequences < 4 ranks) executed rank by rank on one
    GPU through the partitioner's local packing equals one full call."""
    from flashinfer_bench_tma_thrust_b200 import partition as PT
    x = W.prefill_inputs([300, 0, 77], seed=41)
    xd = to_dev(x)
    ref_out, ref_state = prefill.kernel(*xd.args())
    plan = PT.plan_prefill(x.lengths, 4, 16, 32)
    assert plan.groups > 1
    parts = [PT.run_prefill_local(plan, r, prefill.kernel, *xd.args()) for r in range(4)]
    out, state = PT.assemble_prefill(parts, x.q.shape[0], 3, 32, x.cu_seqlens)
    assert_out_close(out, ref_out, "partitioned vs full")
    assert_state_close(state, ref_state, PREFILL_STATE_ATOL, "partitioned vs full")


def test_chunked_flags_bad_cu_seqlens_without_faulting():
    """cu_seqlens outside [0, T] is used clamped and flagged (status bit 1); overlapping
    ranges whose chunks would overflow the two-phase workspace are flagged and compute
    nothing (states passed through) — no access leaves the workspace or the tensors."""
    x = to_dev(W.prefill_inputs([640], HQ=2, HV=4, seed=5))
    prefill.reset_device_status()
    args = list(x.args())
    # overlap: sequences [0, 640), (640 -> 0: empty), [0, 640): 20 chunks > 10 + 3 capacity
    args[8] = torch.tensor([0, 640, 0, 640], dtype=torch.int32, device="cuda")
    state = torch.randn(3, 4, 128, 128, device="cuda")
    args[3] = state
    out, ns = prefill.kernel(*args)
    torch.cuda.synchronize()
    assert prefill.device_status() & 2
    assert torch.equal(ns, state)
    prefill.reset_device_status()
    # out of range: [0, 700) with T = 640 is clamped to [0, 640)
    args[8] = torch.tensor([0, 700], dtype=torch.int64, device="cuda")
    args[3] = x.state
    out, ns = prefill.kernel(*args)
    ref_out, ref_ns = prefill.kernel(*x.args())
    torch.cuda.synchronize()
    assert prefill.device_status() & 2
    assert torch.equal(out, ref_out) and torch.equal(ns, ref_ns)
    prefill.reset_device_status()
    prefill.kernel(*x.args())
    assert prefill.device_status() == 0
