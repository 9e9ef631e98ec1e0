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
