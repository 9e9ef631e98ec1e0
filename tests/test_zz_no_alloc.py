"""The allocation-free chunked prefill entry point (gdn_prefill_chunked_fwd_noalloc).

It exists for callers that cannot hand the library device memory — an engine
whose memory pool owns the device and forbids allocations mid-step, or an FFI
caller with no CUDA allocator — and uses a fixed scratch array compiled into the
library instead of a caller workspace. This test calls it through the C ABI
twice in a row (the second call sees the scratch the first one left behind) and
checks both results against the regular entry point, within the parity
tolerances used by every GPU test. Kept in its own file, collected last.
"""
import pytest
import torch

from flashinfer_bench_tma_thrust_b200 import _lib, prefill, workloads as W
from parity import PREFILL_STATE_ATOL, assert_out_close, assert_state_close, to_dev

pytestmark = pytest.mark.gpu


def _call_noalloc(P):
    lib = _lib.load()
    out = torch.empty(P.T, P.HV, P.D, dtype=torch.bfloat16, device=P.dev)
    new_state = torch.empty(P.N, P.HV, P.D, P.D, dtype=torch.float32, device=P.dev)
    rc = lib.gdn_prefill_chunked_fwd_noalloc(
        P.q.data_ptr(), P.k.data_ptr(), P.v.data_ptr(),
        None if P.state is None else P.state.data_ptr(),
        P.A.data_ptr(), P.A_t, P.a.data_ptr(), P.a_t, P.d.data_ptr(), P.d_t, P.b.data_ptr(),
        P.b_t, P.cu.data_ptr(), P.cu_t, P.scale, out.data_ptr(), new_state.data_ptr(),
        P.T, P.N, P.HQ, P.HV, P.D, torch.cuda.current_stream(P.dev).cuda_stream)
    _lib.check(rc, "gdn_prefill_chunked_fwd_noalloc")
    return out, new_state


def test_noalloc_matches_regular_entry_two_calls():
    x = to_dev(W.prefill_inputs([130, 0, 70, 1], HQ=4, HV=8, seed=77))
    ref_out, ref_state = prefill.kernel(*x.args())
    P = prefill.prepare(*x.args())
    for _ in range(2):
        out, new_state = _call_noalloc(P)
        torch.cuda.synchronize()
        assert_out_close(out, ref_out, "noalloc vs chunked")
        assert_state_close(new_state, ref_state, PREFILL_STATE_ATOL, "noalloc vs chunked")
