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


def test_bench_prefill_plans_cover_every_unit_once():
    """The bench's multi-GPU prefill legs: varlen = the configuration's 8 sequences split
    over the ranks (2 head groups per sequence at 8 ranks), long = 4 sequences of 32768
    tokens per rank (whole sequences); every (sequence, v-head) pair lands on one rank."""
    import bench
    for world in (1, 2, 4, 8):
        for workload in ("prefill_varlen", "prefill_long"):
            lengths, with_state, scaling, plan = bench.prefill_plan(workload, world)
            seen = {}
            for r in range(world):
                for u in plan.ranks[r]:
                    for h in range(u.h0, u.h1):
                        assert (u.seq, h) not in seen
                        seen[(u.seq, h)] = r
            assert len(seen) == len(lengths) * 32
            if workload == "prefill_long":
                assert len(lengths) == 4 * world and plan.groups == 1 and scaling == "weak"
                assert all(len(plan.ranks[r]) == 4 for r in range(world))
            else:
                assert len(lengths) == 8 and scaling == "strong" and with_state
    assert bench.prefill_plan("prefill_varlen", 8)[3].groups == 2
