"""Host-side logic of the prefill wrapper that needs no GPU."""
import torch

from flashinfer_bench_tma_thrust_b200 import prefill


def test_workspace_growth_keeps_sticky_status_bits():
    """Growing the per-device workspace keeps the status word set so far (a failure of
    an earlier call is not lost when a larger call replaces the buffer)."""
    dev = torch.device("cpu")
    prefill._workspaces.pop((dev.type, dev.index), None)
    ws = prefill.workspace(dev, 256)
    ws[:4].view(torch.int32)[0] = 3
    grown = prefill.workspace(dev, 1 << 16)
    assert grown.numel() == 1 << 16 and grown.data_ptr() != ws.data_ptr()
    assert int(grown[:4].view(torch.int32)[0]) == 3
    assert prefill.workspace(dev, 1024) is grown  # never shrunk
    prefill._workspaces.pop((dev.type, dev.index), None)
