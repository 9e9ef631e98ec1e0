"""Known-answer test of the tcgen05 path (descriptors, MMA, TMEM load) that the
chunked prefill kernel is built from, against a torch matmul."""
import ctypes

import pytest
import torch

from flashinfer_bench_tma_thrust_b200 import _lib

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("a_mn,b_mn", [(0, 0), (0, 1), (1, 0), (1, 1)])
def test_umma_gemm_128x64x128(a_mn, b_mn):
    lib = _lib.load()
    g = torch.Generator().manual_seed(a_mn * 2 + b_mn)
    A = torch.randn(128, 128, generator=g).to(torch.bfloat16).cuda()
    B = torch.randn(128, 64, generator=g).to(torch.bfloat16).cuda()
    D = torch.full((128, 64), float("nan"), device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = lib.gdn_selftest_umma(A.data_ptr(), B.data_ptr(), D.data_ptr(), a_mn, b_mn,
                               status.data_ptr(), torch.cuda.current_stream().cuda_stream)
    _lib.check(rc, "gdn_selftest_umma")
    torch.cuda.synchronize()
    assert status.item() == 0, "MMA completion wait timed out"
    ref = A.float() @ B.float()
    assert torch.allclose(D, ref, atol=1e-3, rtol=1e-4), (D - ref).abs().max().item()


def test_bounded_wait_gives_up_and_context_survives():
    """A wait on an mbarrier phase that never completes returns after ~1 s with an
    error status (no hang, no trap); the GPU context keeps working afterwards."""
    lib = _lib.load()
    status = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    waited = torch.zeros(1, dtype=torch.int64, device="cuda")
    rc = lib.gdn_selftest_wait_timeout(status.data_ptr(), waited.data_ptr(),
                                       torch.cuda.current_stream().cuda_stream)
    _lib.check(rc, "gdn_selftest_wait_timeout")
    torch.cuda.synchronize()
    assert status.item() == 1
    assert 0.9e9 <= waited.item() <= 5e9, waited.item()
    x = torch.ones(1024, device="cuda")  # the context is still usable
    assert (x * 2).sum().item() == 2048


def test_umma_a_from_tmem_128x128x128():
    """tcgen05.mma with A read from tensor memory (the form of the transposed products)."""
    lib = _lib.load()
    g = torch.Generator().manual_seed(5)
    A = torch.randn(128, 128, generator=g).to(torch.bfloat16).cuda()
    B = torch.randn(128, 128, generator=g).to(torch.bfloat16).cuda()
    D = torch.full((128, 128), float("nan"), device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = lib.gdn_selftest_umma_ts(A.data_ptr(), B.data_ptr(), D.data_ptr(), status.data_ptr(),
                                  torch.cuda.current_stream().cuda_stream)
    _lib.check(rc, "gdn_selftest_umma_ts")
    torch.cuda.synchronize()
    assert status.item() == 0
    ref = A.float() @ B.float()
    assert torch.allclose(D, ref, atol=1e-3, rtol=1e-4), (D - ref).abs().max().item()
