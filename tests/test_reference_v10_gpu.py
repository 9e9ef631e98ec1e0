"""The reference's own GPU decode kernel ("v10", gdn/kernels/cute_cpp/gdn_decode_v10.cuh,
built by oracle/build_ref.py into oracle/_ref/ where the reference checkout exists) as
a second comparator for the decode kernel here, at the 16/32-head configuration.

* With BLOCK_V = 16 and 32 (the reference's choice for B <= 16 and B <= 128,
  gdn/decode/solution/cuda/kernel.py:484-490) it computes the same decode step: our
  outputs and states agree with it within the parity tolerances (it uses the fast
  __expf / __logf gate arithmetic, so it is not bit-identical).
* With BLOCK_V = 64 (the reference's choice for B > 128, hence for the B = 256
  benchmark configuration) its launcher asks for 67 KB of dynamic shared memory
  without raising the kernel's 48 KB default limit, so the launch is rejected
  (cudaErrorInvalidValue) and nothing is computed."""
import pytest
import torch

from flashinfer_bench_tma_thrust_b200 import decode, workloads as W
from oracle import ref_v10
from parity import DECODE_STATE_ATOL, assert_out_close, assert_state_close

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not ref_v10.available(), reason="reference comparator not built")]


@pytest.mark.parametrize("variant", [0, 1])
@pytest.mark.parametrize("B,block_v", [(4, 16), (64, 32), (256, 32)])
def test_reference_v10_matches_ours(B, block_v, variant):
    x = W.decode_inputs(B, seed=500 + B, gen_device="cuda", device="cuda")
    out_r = torch.empty(B, 32, 128, dtype=torch.bfloat16, device="cuda")
    ns_r = torch.empty_like(x.state)
    rc = ref_v10.decode(x.q, x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b, out_r, ns_r,
                        x.scale, block_v, variant)
    torch.cuda.synchronize()
    assert rc == 0
    out, ns = decode.kernel(*x.args())
    assert_out_close(out[:, 0], out_r, f"ours vs reference v10, B={B}")
    assert_state_close(ns, ns_r, DECODE_STATE_ATOL, f"ours vs reference v10, B={B}")


def test_reference_v10_block_v64_launch_is_rejected():
    """The B > 128 configuration of the reference's packaged CUDA decode does not run."""
    B = 256
    x = W.decode_inputs(B, seed=7, gen_device="cuda", device="cuda")
    out_r = torch.full((B, 32, 128), 7.0, dtype=torch.bfloat16, device="cuda")
    ns_r = torch.full_like(x.state, 7.0)
    rc = ref_v10.decode(x.q, x.k, x.v, x.state, x.A_log, x.a, x.dt_bias, x.b, out_r, ns_r,
                        x.scale, 64, 0)
    torch.cuda.synchronize()
    assert rc != 0
    assert bool((ns_r == 7.0).all()) and bool((out_r == 7.0).all())
