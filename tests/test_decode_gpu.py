"""Decode parity on the GPU: the sm_100a kernel (through the C ABI) vs the oracle
and vs the reference's golden outputs."""
import pytest
import torch

from flashinfer_bench_tma_thrust_b200 import decode, workloads as W
from golden import golden
from oracle import gdn_oracle
from parity import (DECODE_STATE_ATOL, assert_out_close, assert_state_close, to_dev,
                    state_errors, STATE_REL_FROB)

pytestmark = pytest.mark.gpu

DEC_CASES = [c for c in golden.case_names() if c.startswith("dec_")]


@pytest.mark.parametrize("name", DEC_CASES)
def test_decode_matches_reference_golden(name):
    _, x, exp = golden.load_case(name)
    out, ns = decode.kernel(*to_dev(x).args())
    assert_out_close(out, exp["out"], name)
    err, rel = golden.compare_state(ns, exp, atol=DECODE_STATE_ATOL, rtol_frob=STATE_REL_FROB)
    assert err <= DECODE_STATE_ATOL and rel <= STATE_REL_FROB, (name, err, rel)


@pytest.mark.parametrize("B", [1, 2, 4, 16, 64, 256])
def test_decode_full_heads_vs_oracle(B):
    x = W.decode_inputs(B, seed=100 + B)
    ref_out, ref_ns = gdn_oracle.decode(*x.args())
    out, ns = decode.kernel(*to_dev(x).args())
    assert out.shape == (B, 1, 32, 128) and out.dtype == torch.bfloat16
    assert ns.shape == (B, 32, 128, 128) and ns.dtype == torch.float32
    assert_out_close(out, ref_out, f"B={B}")
    assert_state_close(ns, ref_ns, DECODE_STATE_ATOL, f"B={B}")


@pytest.mark.parametrize("B,HQ,HV", [(1, 4, 8), (4, 4, 8), (16, 4, 8), (64, 4, 8), (3, 2, 8)])
def test_decode_reference_test_distribution(B, HQ, HV):
    """The reference's decode test setup (gdn/tests/test_correctness.py:193-240): unit
    normal state, fp32 gates, qk4/v8 heads; plus a GVA ratio of 4."""
    g = torch.Generator().manual_seed(42)
    D = 128
    q = torch.randn(B, 1, HQ, D, generator=g).to(torch.bfloat16)
    k = torch.randn(B, 1, HQ, D, generator=g).to(torch.bfloat16)
    v = torch.randn(B, 1, HV, D, generator=g).to(torch.bfloat16)
    state = torch.randn(B, HV, D, D, generator=g)
    A_log = torch.randn(HV, generator=g)
    a = torch.randn(B, 1, HV, generator=g)
    dt_bias = torch.randn(HV, generator=g)
    b = torch.randn(B, 1, HV, generator=g)
    args = (q, k, v, state, A_log, a, dt_bias, b, 1.0 / D ** 0.5)
    ref_out, ref_ns = gdn_oracle.decode(*args)
    out, ns = decode.kernel(*[t.cuda() if isinstance(t, torch.Tensor) else t for t in args])
    # outputs reach |o| ~ 4 here, where one bf16 ulp is 0.0156: use atol + rtol 1e-2
    # (the reference's absolute 1e-2, test_correctness.py:240, is below one ulp at that
    # magnitude); the state keeps the reference's absolute 1e-4 at unit-scale state
    assert_out_close(out, ref_out, f"B={B}")
    err, rel = state_errors(ns, ref_ns)
    assert err < 1e-4 and rel < STATE_REL_FROB


def test_decode_no_state_and_bf16_dt_bias():
    x = W.decode_inputs(8, seed=7, with_state=False)
    xd = to_dev(x)
    xd.dt_bias = xd.dt_bias.to(torch.bfloat16)
    xd.A_log = xd.A_log.to(torch.bfloat16)
    x.dt_bias = x.dt_bias.to(torch.bfloat16).float()
    x.A_log = x.A_log.to(torch.bfloat16).float()
    ref_out, ref_ns = gdn_oracle.decode(*x.args())
    out, ns = decode.kernel(*xd.args())
    assert_out_close(out, ref_out)
    assert_state_close(ns, ref_ns, DECODE_STATE_ATOL)


def test_decode_inputs_not_modified_and_inplace_variant():
    x = to_dev(W.decode_inputs(16, seed=9))
    s0 = x.state.clone()
    out, ns = decode.kernel(*x.args())
    assert torch.equal(x.state, s0), "kernel() must not modify its state input"
    st = x.state.clone()
    out2, st_ret = decode.kernel_inplace(x.q, x.k, x.v, st, x.A_log, x.a, x.dt_bias, x.b, x.scale)
    assert st_ret.data_ptr() == st.data_ptr()
    assert torch.equal(out2, out) and torch.equal(st, ns)


def test_decode_scale_default():
    x = to_dev(W.decode_inputs(2, seed=11))
    o1, _ = decode.kernel(*x.args()[:-1], None)
    o2, _ = decode.kernel(*x.args()[:-1], 0.0)
    o3, _ = decode.kernel(*x.args()[:-1], 1.0 / 128 ** 0.5)
    assert torch.equal(o1, o3) and torch.equal(o2, o3)


def test_decode_large_batch_64bit_offsets():
    """B=4096 at 32 v-heads puts state offsets past 2^31 elements (the reference kernels
    index with 32-bit ints, gdn/kernels/cute_cpp/gdn_decode_v10.cuh:228). Checked on
    sampled batch rows, the rows being independent."""
    B = 4096
    x = W.decode_inputs(B, seed=13, gen_device="cuda", device="cuda")
    out, ns = decode.kernel(*x.args())
    for bi in (0, 1, 2047, 4094, 4095):
        sl = lambda t: t[bi:bi + 1]  # noqa: E731
        ref_out, ref_ns = gdn_oracle.decode(sl(x.q).cpu(), sl(x.k).cpu(), sl(x.v).cpu(),
                                            sl(x.state).cpu(), x.A_log.cpu(), sl(x.a).cpu(),
                                            x.dt_bias.cpu(), sl(x.b).cpu(), x.scale)
        assert_out_close(out[bi:bi + 1], ref_out, f"b={bi}")
        assert_state_close(ns[bi:bi + 1], ref_ns, DECODE_STATE_ATOL, f"b={bi}")
    del ns, out, x
    torch.cuda.empty_cache()


def test_decode_rejects_bad_inputs():
    x = to_dev(W.decode_inputs(2, seed=1))
    with pytest.raises(ValueError):
        decode.kernel(x.q, x.k, x.v[:, :, :5], x.state, x.A_log, x.a, x.dt_bias, x.b, x.scale)
    with pytest.raises(ValueError):
        decode.kernel(x.q.cpu(), x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b, x.scale)
    with pytest.raises(TypeError):
        decode.kernel(x.q.float(), x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b, x.scale)


@pytest.mark.parametrize("T", [2, 7, 65])
def test_multitoken_decode_equals_consecutive_steps(T):
    """T tokens per sequence in one call == T single-token decode steps (oracle)."""
    B = 3
    g = torch.Generator().manual_seed(T)
    x = W.decode_inputs(B, seed=T)
    q = torch.nn.functional.normalize(torch.randn(B, T, 16, 128, generator=g), dim=-1).to(torch.bfloat16)
    k = torch.nn.functional.normalize(torch.randn(B, T, 16, 128, generator=g), dim=-1).to(torch.bfloat16)
    v = torch.randn(B, T, 32, 128, generator=g).to(torch.bfloat16)
    a = torch.randn(B, T, 32, generator=g).to(torch.bfloat16)
    b = torch.randn(B, T, 32, generator=g).to(torch.bfloat16)
    s = x.state
    ref_outs = []
    for t in range(T):
        o, s = gdn_oracle.decode(q[:, t:t + 1], k[:, t:t + 1], v[:, t:t + 1], s, x.A_log,
                                 a[:, t:t + 1], x.dt_bias, b[:, t:t + 1], x.scale)
        ref_outs.append(o)
    ref_out = torch.cat(ref_outs, dim=1)
    dv = lambda t: t.cuda()  # noqa: E731
    out, ns = decode.kernel_multitoken(dv(q), dv(k), dv(v), dv(x.state), dv(x.A_log), dv(a),
                                       dv(x.dt_bias), dv(b), x.scale)
    assert out.shape == (B, T, 32, 128)
    assert_out_close(out, ref_out, f"T={T}")
    assert_state_close(ns, s, DECODE_STATE_ATOL * 5, f"T={T}")
