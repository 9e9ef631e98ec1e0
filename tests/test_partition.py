"""Multi-GPU partitioner (flashinfer_bench_tma_thrust_b200/partition.py) on CPU.

The host logic — planning, local packing, status exchange, reassembly — runs
here as 2 gloo ranks with the CPU oracle standing in for the per-rank operator
(the GPU operator itself is covered by the gpu tests); the distributed result
must equal the single-process oracle on the same inputs. A rank whose compute
raises must make both ranks raise PartitionError instead of hanging.
"""
import os
import socket
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from flashinfer_bench_tma_thrust_b200 import partition as PT, workloads as W
from oracle import gdn_oracle


def test_plan_decode_contiguous_balanced():
    for B, world in [(256, 1), (256, 8), (1000, 8), (3, 8), (0, 2)]:
        sl = PT.plan_decode(B, world)
        assert sl[0][0] == 0 and sl[-1][1] == B
        assert all(a[1] == b[0] for a, b in zip(sl, sl[1:]))
        sizes = [b - a for a, b in sl]
        assert max(sizes) - min(sizes) <= 1


@pytest.mark.parametrize("lengths,world", [
    ([32768] * 32, 8),          # long config: 4 sequences per GPU, whole heads
    ([2641, 2501, 1405, 3002, 2670, 3056, 3789, 615], 8),   # varlen: splits heads
    ([100], 4), ([0, 0, 5], 2), ([7, 0, 19, 3], 3),
])
def test_plan_prefill_covers_every_unit_once(lengths, world):
    HQ, HV = 16, 32
    plan = PT.plan_prefill(lengths, world, HQ, HV)
    seen = {}
    for r in range(world):
        for u in plan.ranks[r]:
            for h in range(u.h0, u.h1):
                assert (u.seq, h) not in seen
                seen[(u.seq, h)] = r
            assert u.h0 % (HV // HQ) == 0 and u.h1 % (HV // HQ) == 0  # whole q/k heads
    assert len(seen) == len(lengths) * HV
    loads = [plan.load(r) for r in range(world)]
    costs = [u.cost for r in range(world) for u in plan.ranks[r]]
    # LPT bound: no rank exceeds the average by more than the largest unit
    assert max(loads) <= sum(loads) / world + max(costs + [0])


def test_plan_long_config_is_four_sequences_per_gpu():
    plan = PT.plan_prefill([32768] * 32, 8, 16, 32)
    assert plan.groups == 1
    assert all(len(plan.ranks[r]) == 4 for r in range(8))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_path, fail_rank):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        x = W.prefill_inputs([70, 0, 33, 5, 128], HQ=2, HV=4, seed=11)
        plan = PT.plan_prefill(x.lengths, world, 2, 4)

        def compute(*args):
            if rank == fail_rank:
                raise RuntimeError("injected failure")
            return gdn_oracle.prefill(*args)

        try:
            res = PT.run_prefill_local(plan, rank, compute, *x.args())
            status = "ok"
        except PT.PartitionError:
            status = "partition_error"
            res = None
        if status == "ok":
            got = PT.gather_prefill(res, x.q.shape[0], len(x.lengths), 4, x.cu_seqlens)
        else:
            got = None
        if rank == 0:
            torch.save({"status": status, "got": got}, out_path)
        else:
            torch.save({"status": status}, out_path + f".{rank}")
    finally:
        dist.destroy_process_group()


def _run(world, fail_rank):
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "out.pt")
        mp.spawn(_worker, args=(world, _free_port(), path, fail_rank), nprocs=world, join=True)
        res0 = torch.load(path)
        others = [torch.load(path + f".{r}") for r in range(1, world)]
    return res0, others


def test_distributed_prefill_equals_single_process():
    res0, others = _run(2, fail_rank=-1)
    assert res0["status"] == "ok" and all(o["status"] == "ok" for o in others)
    x = W.prefill_inputs([70, 0, 33, 5, 128], HQ=2, HV=4, seed=11)
    ref_out, ref_state = gdn_oracle.prefill(*x.args())
    out, state = res0["got"]
    assert torch.equal(out, ref_out)
    assert torch.allclose(state, ref_state, atol=1e-6, rtol=0)


def test_failed_rank_raises_on_every_rank():
    res0, others = _run(2, fail_rank=1)
    assert res0["status"] == "partition_error"
    assert all(o["status"] == "partition_error" for o in others)


def test_decode_sharding_matches_full_batch():
    x = W.decode_inputs(5, HQ=2, HV=4, seed=3)
    ref_out, ref_state = gdn_oracle.decode(*x.args())
    slices = PT.plan_decode(5, 3)
    outs, states = [], []
    for r in range(3):
        o, s = gdn_oracle.decode(*PT.decode_local(slices, r, *x.args()))
        outs.append(o)
        states.append(s)
    assert torch.equal(torch.cat(outs), ref_out)
    assert torch.allclose(torch.cat(states), ref_state, atol=1e-7, rtol=0)
