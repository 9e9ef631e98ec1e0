"""Prefill parity on the GPU: chunked (kernel) and token-sequential (kernel_recurrent)
sm_100a kernels through the C ABI vs the oracle and the reference's golden outputs."""
import pytest
import torch

from flashinfer_bench_tma_thrust_b200 import prefill, workloads as W
from golden import golden
from oracle import gdn_oracle
from parity import (PREFILL_STATE_ATOL, STATE_REL_FROB, assert_out_close, assert_state_close,
                    state_errors, to_dev)

pytestmark = pytest.mark.gpu

PRE_CASES = [c for c in golden.case_names() if c.startswith("pre_")]
IMPLS = {"chunked": prefill.kernel, "fused": prefill.kernel_fused,
         "recurrent": prefill.kernel_recurrent}


def _report(name, out, ref_out, ns, ref_ns, extra=None):
    """Append the parity figures of a full-size case to $GDN_PARITY_REPORT (JSON lines)
    when that variable names a file; the assertions do not depend on it."""
    import json
    import os
    path = os.environ.get("GDN_PARITY_REPORT")
    if not path:
        return
    o, r = out.detach().float().cpu(), ref_out.detach().float().cpu()
    err, rel = state_errors(ns, ref_ns)
    rec = {"case": name, "out_max_abs": (o - r).abs().max().item(),
           "out_rel_frob": ((o - r).norm() / r.norm().clamp_min(1e-30)).item(),
           "state_max_abs": err, "state_rel_frob": rel}
    rec.update(extra or {})
    with open(path, "a") as f:
        f.write(json.dumps(rec) + "\n")


# ---- the benchmark configurations against the CPU oracle (first in this file) ---------
def test_chunked_vs_oracle_varlen_config():
    """Config 4 in full: 8 sequences with lengths ~U[512, 4096] (seed 0), int32
    cu_seqlens, initial state N(0, 0.02), 16/32 heads; the chunked kernel (and the fused
    single-kernel path) against the CPU oracle (the reference's PyTorch recurrence,
    restated) on the same inputs. The oracle takes a few seconds per 10K tokens."""
    lengths = W.varlen_lengths(seed=0)
    x = W.prefill_inputs(lengths, seed=0, cu_dtype=torch.int32)
    assert x.cu_seqlens.dtype == torch.int32 and x.state is not None
    ref_out, ref_ns = gdn_oracle.prefill(*x.args())
    xd = to_dev(x)
    for name, fn in (("chunked", prefill.kernel), ("fused", prefill.kernel_fused)):
        out, ns = fn(*xd.args())
        torch.cuda.synchronize()
        _report(f"varlen_config_{name}", out, ref_out, ns, ref_ns, {"T": sum(lengths)})
        assert_out_close(out, ref_out, f"varlen config, {name} vs oracle")
        assert_state_close(ns, ref_ns, PREFILL_STATE_ATOL, f"varlen config, {name} vs oracle")
    assert prefill.device_status() == 0


SLOW_LENGTHS = [[1000, 130, 0, 2048, 64], [129, 192, 193, 256], [4097]]


@pytest.mark.parametrize("impl", sorted(IMPLS))
@pytest.mark.parametrize("lengths", SLOW_LENGTHS, ids=lambda l: "-".join(map(str, l)))
def test_prefill_slow_decay_vs_oracle(lengths, impl):
    """Gates with slow decay (g ~ 0.98 per token: the state carries across many 64-token
    chunks; with the benchmark's gates it decays to zero in fp32 within one chunk, so
    the inter-chunk state products would go untested), initial state N(0, 0.02)."""
    x = W.prefill_inputs(lengths, seed=len(lengths) + 7, dist="slowdecay")
    ref_out, ref_ns = gdn_oracle.prefill(*x.args())
    out, ns = IMPLS[impl](*to_dev(x).args())
    torch.cuda.synchronize()
    _report(f"slowdecay_{impl}_{'-'.join(map(str, lengths))}", out, ref_out, ns, ref_ns)
    assert_out_close(out, ref_out, f"slow decay {lengths}, {impl}")
    assert_state_close(ns, ref_ns, PREFILL_STATE_ATOL, f"slow decay {lengths}, {impl}")


def test_prefill_slow_decay_split_call_vs_oracle(monkeypatch):
    """Slow-decay gates through the split-call path (4 x 8192 tokens, 32 v-heads: the
    second scan part starts from the states the first wrote, which now matter), against
    the oracle on the first and the last sequence."""
    monkeypatch.delenv("GDN_PREFILL_OVERLAP", raising=False)
    lengths = [8192] * 4
    x = W.prefill_inputs(lengths, seed=11, dist="slowdecay")
    if prefill.launches_per_call(4, sum(lengths), 32) != 6:
        pytest.skip("no split call on this GPU for these sizes")
    out, ns = prefill.kernel(*to_dev(x).args())
    torch.cuda.synchronize()
    for n in (0, 3):
        xs, s0, e0 = _seq_slice(x, n)
        ref_out, ref_ns = gdn_oracle.prefill(*xs.args())
        _report(f"slowdecay_split_seq{n}", out[s0:e0], ref_out, ns[n:n + 1], ref_ns)
        assert_out_close(out[s0:e0], ref_out, f"slow decay split, sequence {n}")
        assert_state_close(ns[n:n + 1], ref_ns, PREFILL_STATE_ATOL,
                           f"slow decay split, sequence {n}")


def _seq_slice(x, n):
    """Inputs of sequence n of a packed prefill input alone (cu_seqlens [0, L])."""
    import dataclasses
    cu = [int(c) for c in x.cu_seqlens.tolist()]
    s, e = cu[n], cu[n + 1]
    vals = {f.name: getattr(x, f.name) for f in dataclasses.fields(x)}
    for key in ("q", "k", "v", "a", "b"):
        vals[key] = vals[key][s:e]
    vals["cu_seqlens"] = torch.tensor([0, e - s], dtype=x.cu_seqlens.dtype)
    if vals["state"] is not None:
        vals["state"] = vals["state"][n:n + 1]
    return type(x)(**vals), s, e


def test_chunked_vs_oracle_long_config_split(monkeypatch):
    """Config 5's 1-GPU run in full (4 sequences x 32768 tokens, zero initial state,
    16/32 heads), through the split-call path (128 scan chains leave SMs idle, so the
    prep of each sequence's late chunks overlaps the scan: asserted through the
    library's launch count), against the CPU oracle on the first and the last sequence
    (the oracle costs ~10 s per 32768 tokens; every sequence runs the same code)."""
    monkeypatch.delenv("GDN_PREFILL_OVERLAP", raising=False)
    lengths = [32768] * 4
    x = W.prefill_inputs(lengths, seed=2000, with_state=False)
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    if sms - 4 * 32 >= 8:
        assert prefill.launches_per_call(4, sum(lengths), 32) == 6, "call not split"
    out, ns = prefill.kernel(*to_dev(x).args())
    torch.cuda.synchronize()
    for n in (0, 3):
        xs, s, e = _seq_slice(x, n)
        ref_out, ref_ns = gdn_oracle.prefill(*xs.args())
        _report(f"long_config_seq{n}", out[s:e], ref_out, ns[n:n + 1], ref_ns, {"T": e - s})
        assert_out_close(out[s:e], ref_out, f"long config, sequence {n} vs oracle")
        assert_state_close(ns[n:n + 1], ref_ns, PREFILL_STATE_ATOL,
                           f"long config, sequence {n} vs oracle")
    assert prefill.device_status() == 0



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
    monkeypatch.setenv("GDN_PREFILL_OVERLAP", "1")
    if prefill.launches_per_call(4, 4 * 8192, 32) != 6:
        pytest.skip("this GPU leaves fewer than 8 SMs idle for 128 chains: no split call")
    monkeypatch.setenv("GDN_PREFILL_OVERLAP", "0")
    assert prefill.launches_per_call(4, 4 * 8192, 32) == 4
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
    ref_out, ref_ns = prefill.kernel(*x.args())
    args[8] = torch.tensor([0, 700], dtype=torch.int64, device="cuda")
    args[3] = x.state
    out, ns = prefill.kernel(*args)
    torch.cuda.synchronize()
    assert prefill.device_status() & 2
    assert torch.equal(out, ref_out) and torch.equal(ns, ref_ns)
    prefill.reset_device_status()
    prefill.kernel(*x.args())
    assert prefill.device_status() == 0


def test_chunked_failure_raises_through_python_entry():
    """A failure the kernels report in the status word reaches the caller: with
    check=True the failing call raises GDNError; without it the next call on the device
    raises; reset_device_status() clears it, and a grown workspace keeps the bits."""
    from flashinfer_bench_tma_thrust_b200._lib import GDNError
    x = to_dev(W.prefill_inputs([640], HQ=2, HV=4, seed=5))
    prefill.reset_device_status()
    torch.cuda.synchronize()
    # start from a fresh (small) workspace so that the big call below really grows it
    prefill._workspaces.pop(("cuda", torch.cuda.current_device()), None)
    args = list(x.args())
    args[8] = torch.tensor([0, 700], dtype=torch.int64, device="cuda")  # T = 640
    with pytest.raises(GDNError, match="status bits 0x2"):
        prefill.kernel(*args, check=True)
    with pytest.raises(GDNError):
        prefill.kernel(*x.args())
    prefill.reset_device_status()
    prefill.kernel(*x.args(), check=True)
    # a larger call grows the workspace: the sticky bit set before it survives
    prefill.kernel(*args)
    torch.cuda.synchronize()
    big = to_dev(W.prefill_inputs([4096, 4096], HQ=2, HV=4, seed=6))
    with pytest.raises(GDNError):
        prefill.kernel(*big.args(), check=True)
    assert prefill.device_status() & 2
    prefill.reset_device_status()
    prefill.kernel(*big.args(), check=True)
    assert prefill.device_status() == 0


@pytest.mark.parametrize("path", ["two_phase", "fused"])
def test_split_calls_from_two_host_threads(path):
    """Two host threads call the C ABI at the same time on their own streams and
    workspaces, every result compared bit for bit with the single-threaded one. Two-phase
    path: split-call sizes (4 x 8192 tokens, 32 v-heads; the side stream and its events
    are shared per device). Fused path (a 256-byte workspace): the same inputs. Timing
    differences between concurrent calls expose hand-off races inside a kernel."""
    import threading
    from flashinfer_bench_tma_thrust_b200 import _checks as C, _lib
    if path == "two_phase" and prefill.launches_per_call(4, 4 * 8192, 32) != 6:
        pytest.skip("no split call on this GPU for these sizes")
    lib = _lib.load()
    xs = [W.prefill_inputs([8192] * 4, seed=90 + i, gen_device="cuda", device="cuda")
          for i in range(2)]
    ref_fn = prefill.kernel if path == "two_phase" else prefill.kernel_fused
    refs = [ref_fn(*x.args()) for x in xs]
    torch.cuda.synchronize()
    Ps = [prefill.prepare(*x.args()) for x in xs]
    nb = (lib.gdn_prefill_chunked_workspace_size(Ps[0].T, Ps[0].N, Ps[0].HV)
          if path == "two_phase" else 256)
    wss = [torch.zeros(nb, dtype=torch.uint8, device="cuda") for _ in range(2)]
    streams = [torch.cuda.Stream() for _ in range(2)]
    results = [[None] * 6 for _ in range(2)]
    errors = []
    barrier = threading.Barrier(2)

    def worker(i):
        try:
            P, st = Ps[i], streams[i]
            barrier.wait()
            for r in range(6):
                with torch.cuda.stream(st):
                    out, ns = prefill._alloc_outputs(P)
                rc = lib.gdn_prefill_chunked_fwd(
                    P.q.data_ptr(), P.k.data_ptr(), P.v.data_ptr(), C.ptr(P.state),
                    P.A.data_ptr(), P.A_t, P.a.data_ptr(), P.a_t, P.d.data_ptr(), P.d_t,
                    P.b.data_ptr(), P.b_t, P.cu.data_ptr(), P.cu_t, P.scale, out.data_ptr(),
                    ns.data_ptr(), P.T, P.N, P.HQ, P.HV, P.D, wss[i].data_ptr(), nb,
                    st.cuda_stream)
                _lib.check(rc, "gdn_prefill_chunked_fwd")
                results[i][r] = (out, ns)
        except Exception as e:  # noqa: BLE001 - reported below
            errors.append(e)

    ths = [threading.Thread(target=worker, args=(i,)) for i in range(2)]
    for t in ths:
        t.start()
    for t in ths:
        t.join()
    torch.cuda.synchronize()
    assert not errors, errors
    bad = []
    for i in range(2):
        assert int(wss[i][:4].view(torch.int32).item()) == 0
        for r, (out, ns) in enumerate(results[i]):
            if not (torch.equal(out, refs[i][0]) and torch.equal(ns, refs[i][1])):
                dif = (out != refs[i][0]).any(-1).nonzero()
                bad.append((i, r, (out.float() - refs[i][0].float()).abs().max().item(),
                            (ns - refs[i][1]).abs().max().item(), int(dif.shape[0]),
                            dif[:6].tolist()))
    assert not bad, ("(thread, call, max |out diff|, max |state diff|, differing (token, "
                     f"head) rows, first ones): {bad}")
