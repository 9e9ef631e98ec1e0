"""Multi-GPU partitioner for the GDN operators (one process per GPU).

Every (sequence, v-head) pair of GDN is an independent recurrence: its state,
outputs and gates belong to it alone, and q/k are shared only by the v-heads of
one q/k head. The path therefore shards with no data-path collective:

* decode: contiguous batch slices — each rank owns state[b0:b1] for good;
* prefill: whole sequences, assigned longest-processing-time first on their
  lengths; when there are fewer sequences than ranks (or the longest sequence
  would dominate one rank) the v-heads are split too, in groups that keep the
  v-heads of one q/k head together, so each unit is (sequence, head group).

Each rank builds packed local inputs (local ``cu_seqlens``, its heads only),
runs the single-GPU operator, and reports success to the others through one
tiny all-reduce of a status flag (host-side failure detection: a rank whose
compute raised makes every rank raise ``PartitionError`` instead of hanging at
a later collective). Gathering the outputs to one rank is optional and separate
from the compute (``gather_prefill``); the reference has no multi-GPU code
(its kernels are single-GPU, gdn/benchmarks/bench_modal.py:149).
"""
from __future__ import annotations

import heapq
from dataclasses import dataclass, field

import torch


class PartitionError(RuntimeError):
    """A rank failed; raised on every rank after the status exchange."""


@dataclass(frozen=True)
class Unit:
    seq: int          # sequence index in the global batch
    h0: int           # first v-head (inclusive)
    h1: int           # last v-head (exclusive)
    cost: int         # tokens x heads (load estimate)


@dataclass
class PrefillPlan:
    world: int
    HQ: int
    HV: int
    groups: int                      # head groups per sequence
    ranks: list = field(default_factory=list)   # ranks[r] = list[Unit]

    def load(self, r: int) -> int:
        return sum(u.cost for u in self.ranks[r])


def plan_decode(B: int, world: int) -> list[tuple[int, int]]:
    """Contiguous, balanced batch slices [(b0, b1)] per rank (sizes differ by <= 1)."""
    if world <= 0 or B < 0:
        raise ValueError("world must be positive and B non-negative")
    base, extra = divmod(B, world)
    out, b = [], 0
    for r in range(world):
        n = base + (1 if r < extra else 0)
        out.append((b, b + n))
        b += n
    return out


def _head_groups(N: int, lengths, world: int, HQ: int) -> int:
    """How many head groups to split each sequence into: enough units to occupy every
    rank, and a longest unit no larger than the balanced share, limited by the q/k
    head count (a group holds whole q/k heads)."""
    total = sum(max(0, int(l)) for l in lengths)
    longest = max([max(0, int(l)) for l in lengths] or [0])
    g = 1
    while g < HQ and (N * g < world or (total > 0 and longest / g > total / world)):
        g *= 2
    while HQ % g:
        g //= 2
    return max(1, g)


def plan_prefill(lengths, world: int, HQ: int, HV: int) -> PrefillPlan:
    """Assign (sequence, head-group) units to ranks, longest processing time first."""
    if world <= 0:
        raise ValueError("world must be positive")
    if HV % HQ:
        raise ValueError("HV must be a multiple of HQ")
    lengths = [int(l) for l in lengths]
    N = len(lengths)
    G = _head_groups(N, lengths, world, HQ)
    ratio = HV // HQ
    qh_per_group = HQ // G
    units = []
    for n, L in enumerate(lengths):
        for g in range(G):
            h0 = g * qh_per_group * ratio
            h1 = (g + 1) * qh_per_group * ratio
            units.append(Unit(n, h0, h1, max(0, L) * (h1 - h0)))
    plan = PrefillPlan(world=world, HQ=HQ, HV=HV, groups=G, ranks=[[] for _ in range(world)])
    heap = [(0, r) for r in range(world)]
    for u in sorted(units, key=lambda u: (-u.cost, u.seq, u.h0)):
        load, r = heapq.heappop(heap)
        plan.ranks[r].append(u)
        heapq.heappush(heap, (load + u.cost, r))
    for r in range(world):
        plan.ranks[r].sort(key=lambda u: (u.h0, u.seq))
    return plan


@dataclass
class LocalPrefill:
    """Packed inputs of one rank: runs of units that share a head range are packed
    into one operator call each (one call per distinct head group)."""
    calls: list      # [(h0, h1, seqs, args_tuple)]


def build_local_prefill(plan: PrefillPlan, rank: int, q, k, v, state, A_log, a, dt_bias, b,
                        cu_seqlens, scale, device=None) -> LocalPrefill:
    """Slice the global inputs for `rank`: per head group, pack its sequences' tokens
    and build local cu_seqlens (same dtype as the global one)."""
    cu = [int(x) for x in cu_seqlens.tolist()]
    ratio = plan.HV // plan.HQ
    by_group: dict = {}
    for u in plan.ranks[rank]:
        by_group.setdefault((u.h0, u.h1), []).append(u.seq)
    calls = []
    for (h0, h1), seqs in sorted(by_group.items()):
        seqs = sorted(seqs)
        idx = [torch.arange(max(cu[n], 0), max(cu[n + 1], cu[n], 0)) for n in seqs]
        tok = torch.cat(idx) if idx else torch.zeros(0, dtype=torch.long)
        lens = [len(i) for i in idx]
        lcu = torch.zeros(len(seqs) + 1, dtype=cu_seqlens.dtype)
        if lens:
            lcu[1:] = torch.cumsum(torch.tensor(lens, dtype=torch.int64), 0).to(cu_seqlens.dtype)
        qh0, qh1 = h0 // ratio, h1 // ratio
        dev = device if device is not None else q.device
        mv = lambda x: x.to(dev) if x is not None else None  # noqa: E731
        tok_d = tok.to(q.device)
        args = (mv(q.index_select(0, tok_d)[:, qh0:qh1].contiguous()),
                mv(k.index_select(0, tok_d)[:, qh0:qh1].contiguous()),
                mv(v.index_select(0, tok_d)[:, h0:h1].contiguous()),
                None if state is None else mv(state[seqs][:, h0:h1].contiguous()),
                mv(A_log[h0:h1].contiguous()),
                mv(a.index_select(0, tok_d)[:, h0:h1].contiguous()),
                mv(dt_bias[h0:h1].contiguous()),
                mv(b.index_select(0, tok_d)[:, h0:h1].contiguous()),
                mv(lcu), scale)
        calls.append((h0, h1, seqs, lens, args))
    return LocalPrefill(calls)


def exchange_status(ok: bool, group=None) -> None:
    """All ranks learn whether any rank failed (one int all-reduce). Raise on all
    ranks if one did."""
    import torch.distributed as dist
    if not dist.is_available() or not dist.is_initialized():
        if not ok:
            raise PartitionError("local compute failed")
        return
    backend = dist.get_backend(group)
    dev = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else "cpu"
    flag = torch.tensor([0 if ok else 1], dtype=torch.int32, device=dev)
    dist.all_reduce(flag, op=dist.ReduceOp.MAX, group=group)
    if int(flag.item()):
        raise PartitionError("a rank failed during the partitioned GDN step" if ok
                             else "this rank's compute failed")


def run_prefill_local(plan: PrefillPlan, rank: int, compute, *inputs, device=None):
    """Compute this rank's share: returns [(h0, h1, seqs, lens, out, new_state)].
    `compute` is the single-GPU operator (e.g. ``prefill.kernel``). Exceptions are
    turned into a status exchange so that every rank raises ``PartitionError``."""
    results, ok, err = [], True, None
    try:
        local = build_local_prefill(plan, rank, *inputs, device=device)
        for h0, h1, seqs, lens, args in local.calls:
            out, ns = compute(*args)
            results.append((h0, h1, seqs, lens, out, ns))
    except Exception as e:  # noqa: BLE001 - reported to every rank below
        ok, err = False, e
    try:
        exchange_status(ok)
    except PartitionError as pe:
        raise pe from err
    return results


def assemble_prefill(parts_by_rank, T: int, N: int, HV: int, cu_seqlens, state=None,
                     D: int = 128):
    """Rebuild the global (output [T, HV, D] bf16, new_state [N, HV, D, D] fp32) from
    every rank's results (e.g. after an all_gather_object). Sequences no rank holds
    (impossible for a valid plan) keep zeros."""
    cu = [int(x) for x in cu_seqlens.tolist()]
    out = torch.zeros(T, HV, D, dtype=torch.bfloat16)
    new_state = torch.zeros(N, HV, D, D, dtype=torch.float32)
    for parts in parts_by_rank:
        for h0, h1, seqs, lens, o, ns in parts:
            o, ns = o.cpu(), ns.cpu()
            off = 0
            for i, (n, L) in enumerate(zip(seqs, lens)):
                if L:
                    out[cu[n]:cu[n] + L, h0:h1] = o[off:off + L]
                off += L
                new_state[n, h0:h1] = ns[i]
    return out, new_state


def gather_prefill(results, T: int, N: int, HV: int, cu_seqlens, dst: int = 0, D: int = 128):
    """Collect every rank's results on rank `dst` (outside the compute: outputs stay
    on their owning GPU otherwise). Returns the global tensors on `dst`, None elsewhere."""
    import torch.distributed as dist
    cpu_parts = [(h0, h1, s, l, o.cpu(), ns.cpu()) for h0, h1, s, l, o, ns in results]
    world = dist.get_world_size()
    gathered = [None] * world if dist.get_rank() == dst else None
    dist.gather_object(cpu_parts, gathered, dst=dst)
    if dist.get_rank() != dst:
        return None
    return assemble_prefill(gathered, T, N, HV, cu_seqlens, D=D)


def decode_local(slices, rank: int, q, k, v, state, A_log, a, dt_bias, b, scale):
    """Batch slice of the decode inputs owned by `rank`."""
    b0, b1 = slices[rank]
    sl = lambda x: None if x is None else x[b0:b1]  # noqa: E731
    return (sl(q), sl(k), sl(v), sl(state), A_log, sl(a), dt_bias, sl(b), scale)
