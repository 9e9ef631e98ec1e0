"""Benchmark of the GDN hot path on B200 — prints ONE JSON line (rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W]
                    [--workload decode|decode_fp8|prefill_varlen|prefill_long]
                    [--impl ours|reference]

Workloads (seeded synthetic inputs with the benchmark configurations' shapes and
distributions; the reference's official trace dataset is not available):

* ``decode`` (default, the headline): B=256 sequences per GPU, 16 q/k heads,
  32 v heads, D=128, fp32 state [256,32,128,128] (512 MiB read + 512 MiB
  written per step). Metric: state GB/s = 2*B*HV*D*D*4 / t_step, the
  reference's own formula (gdn/scripts/bench_cuda_real.py:556, :589). A step
  feeds the previous step's new_state back in (a real decode loop); the state
  is larger than L2 so no flush is needed.
* ``prefill_varlen``: 8 sequences, lengths ~U[512,4096] (seed 0), int32 cu_seqlens,
  initial state ~N(0,0.02). Metric: tokens/s. With N GPUs the same 8 sequences are
  split into (sequence, head-group) units over the ranks (strong scaling).
* ``prefill_long``: 4 sequences x 32768 tokens per GPU, zero initial state (32 x 32768
  on 8 GPUs). Metric: tokens/s.
* ``decode_fp8``: the fp8-state option alone (B=256 per GPU), a separately reported
  figure (GB/s of fp8 state + row scales).

The decode run (the default) also reports both prefill configurations, the bf16 and
fp8 state options and the decode batch sweep under ``extra``, each with its own
roofline, clocks, e2e and CPU figures where they apply.

Multi-GPU (torchrun, one process per GPU): the work is split with
flashinfer_bench_tma_thrust_b200.partition (decode: contiguous batch slices; prefill:
longest-processing-time assignment of sequences or (sequence, head-group) units); no
data-path collective; the step time is the max over ranks.

``--impl reference`` times the reference's CPU implementation of the same path (its
PyTorch baseline where staged under baseline/_ref, else the oracle's restatement of
it) on the host cores with all threads: the full B=256 decode batch per step when the
run fits in about 150 s, a stated subsample otherwise.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

HQ, HV, D = 16, 32, 128
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0
L2_BYTES = 126 * 2 ** 20


# ----------------------------------------------------------------------------- env / dist
def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), float(
            d.get("bf16_tflops_sustained", d["bf16_tflops"])), "measured"
    return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, 1400.0, "fallback"


def ncu_traffic(key: str):
    """DRAM bytes per launch of the dominant kernel, from a committed ncu summary
    (a line ``traffic_per_launch[<key>] = <bytes>`` in profiles/*.md)."""
    for f in sorted((ROOT / "profiles").glob("*.md")):
        m = re.search(rf"traffic_per_launch\[{re.escape(key)}\]\s*=\s*([0-9.eE+]+)", f.read_text())
        if m:
            return float(m.group(1))
    return None


class ClockSampler:
    """SM clock and throttle-reason sampling during the timed region: NVML polled from a
    background thread about every millisecond (so that even a few-millisecond region gets
    samples; the first sample is taken before the constructor returns), else nvidia-smi
    at its 50 ms minimum. Reads only; changes no GPU setting."""

    # NVML clock-event reason bits (nvmlClocksEventReason*)
    BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
            "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80}
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, device: torch.device):
        import threading
        self.proc = None
        self.file = None
        self.thread = None
        self.sm, self.reasons, self.max_mhz = [], set(), None
        uuid = str(torch.cuda.get_device_properties(device).uuid)
        self.uuid = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
        try:
            import pynvml
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByUUID(self.uuid)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
            get_reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                getattr(pynvml, "nvmlDeviceGetCurrentClocksThrottleReasons")
            self.stop_flag = threading.Event()
            first = threading.Event()

            def poll():
                while True:
                    self.sm.append(float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)))
                    bits = int(get_reasons(h))
                    for name, bit in self.BITS.items():
                        if bits & bit:
                            self.reasons.add(name)
                    first.set()
                    if self.stop_flag.wait(0.001):
                        break

            self.thread = threading.Thread(target=poll, daemon=True)
            self.thread.start()
            first.wait(5.0)
            return
        except Exception:
            self.thread = None
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.uuid, f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=self.file, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.thread is not None:
            self.stop_flag.set()
            self.thread.join(timeout=5)
            sm = list(self.sm)
            return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.max_mhz,
                    "reasons": sorted(self.reasons), "samples": len(sm), "source": "nvml"}
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.flush()
        rows = [r.split(", ") for r in Path(self.file.name).read_text().splitlines() if r.strip()]
        os.unlink(self.file.name)
        sm, mx, reasons = [], None, set()
        for r in rows:
            if len(r) < 9:
                continue
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
            except ValueError:
                continue
            for name, val in zip(self.NAMES, r[5:9]):
                if val.strip() == "Active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm), "source": "nvidia-smi"}


# ----------------------------------------------------------------------------- workloads
def decode_workload(device, seed, B=256):
    from flashinfer_bench_tma_thrust_b200 import workloads as W
    x = W.decode_inputs(B, seed=seed, gen_device=device, device=device)
    state_bytes = 2 * B * HV * D * D * 4
    io_bytes = (2 * B * HQ * D + B * HV * D) * 2 + B * HV * D * 2 + 2 * B * HV * 2
    return x, {"B": B, "state_bytes": state_bytes, "alg_bytes": state_bytes + io_bytes}


def prefill_lengths(workload):
    from flashinfer_bench_tma_thrust_b200 import workloads as W
    if workload == "prefill_varlen":
        return W.varlen_lengths(seed=0), True
    return [32768] * 4, False


def time_steps(step, K, W, device, world):
    for _ in range(W):
        step()
    torch.cuda.synchronize(device)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize(device)
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(K):
        step()
    end.record()
    end.synchronize()
    torch.cuda.synchronize(device)
    ms = start.elapsed_time(end)
    if world > 1:
        t = torch.tensor([ms], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
        torch.distributed.barrier()
    return ms


def kernel_launch_ms(step, n, device):
    """Average device time of one step's launch, CUDA events on the launching stream."""
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(n)]
    torch.cuda.synchronize(device)
    for s, e in evs:
        s.record()
        step()
        e.record()
    torch.cuda.synchronize(device)
    return statistics.mean(s.elapsed_time(e) for s, e in evs)


def reference_impl(op: str):
    """The reference's own CPU implementation of `op` ("decode" / "prefill"): its pure
    PyTorch baseline gdn/<op>/baseline/triton/kernel.py, staged under baseline/_ref by
    ``__graft_entry__.build()`` where the reference checkout exists ("reference"); else
    the oracle's restatement of that file ("port")."""
    import importlib.util
    f = ROOT / "baseline" / "_ref" / "gdn" / op / "baseline" / "triton" / "kernel.py"
    if f.exists():
        spec = importlib.util.spec_from_file_location(f"_gdn_ref_{op}_baseline", f)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        return mod.kernel, "reference", f"gdn/{op}/baseline/triton/kernel.py (the reference's own)"
    from oracle import gdn_oracle
    return getattr(gdn_oracle, op), "port", f"oracle/gdn_oracle.py:{op} (restatement)"


def cpu_decode_time(B_sample, steps, warmup, seed=1000, min_seconds=0.0):
    """Time `steps` CPU decode steps (more while under `min_seconds`) of the reference
    implementation on the first B_sample sequences of the B=256 workload (all host
    threads)."""
    from flashinfer_bench_tma_thrust_b200 import workloads as W
    fn, kind, where = reference_impl("decode")
    torch.set_num_threads(os.cpu_count() or 1)
    x = W.decode_inputs(256, seed=seed)
    sl = [t[:B_sample] if isinstance(t, torch.Tensor) and t.dim() > 1 else t for t in x.args()]
    for _ in range(warmup):
        fn(*sl)
    t0 = time.perf_counter()
    n = 0
    while n < steps or time.perf_counter() - t0 < min_seconds:
        fn(*sl)
        n += 1
    el = time.perf_counter() - t0
    steps = n
    sb = 2 * B_sample * HV * D * D * 4
    cores = torch.get_num_threads()
    return {"value": sb * steps / el / 1e9, "unit": "GB/s", "cores": cores, "kind": kind,
            "sample": f"{B_sample} of the 256 sequences per step ({'the full workload' if B_sample == 256 else 'subsample'}), "
                      f"{steps} steps in {el:.1f} s; {where}, torch CPU fp32, {cores} threads of "
                      f"{os.cpu_count()} cpus"}, el / steps


def decode_sample_size(steps, warmup, budget_s=150.0):
    """Sequences per CPU step so that warmup + steps finish within about budget_s: the
    full B = 256 when it fits (probe: one step on 32 sequences, cost per sequence taken
    25 % higher for safety)."""
    _, per = cpu_decode_time(32, 1, 0)
    per_seq = 1.25 * per / 32
    fit = int(budget_s / max(1, steps + warmup) / max(per_seq, 1e-6))
    return max(1, min(256, fit))


def cpu_prefill_time(lengths, with_state, steps, warmup, tokens_per_seq=64, seed=2000,
                     min_seconds=0.0):
    """Time the reference implementation's prefill on the first `tokens_per_seq` tokens
    of each sequence of the configuration (same head layout and distributions)."""
    from flashinfer_bench_tma_thrust_b200 import workloads as W
    fn, kind, where = reference_impl("prefill")
    torch.set_num_threads(os.cpu_count() or 1)
    sub = [min(l, tokens_per_seq) for l in lengths]
    x = W.prefill_inputs(sub, seed=seed, with_state=with_state)
    for _ in range(warmup):
        fn(*x.args())
    t0 = time.perf_counter()
    n = 0
    while n < steps or time.perf_counter() - t0 < min_seconds:
        fn(*x.args())
        n += 1
    el = time.perf_counter() - t0
    steps = n
    cores = torch.get_num_threads()
    return {"value": sum(sub) * steps / el, "unit": "tokens/s", "cores": cores, "kind": kind,
            "sample": f"first {tokens_per_seq} tokens of each of the {len(lengths)} sequences "
                      f"({sum(sub)} tokens) per step, {steps} steps in {el:.1f} s; {where}, "
                      f"torch CPU fp32, {cores} threads of {os.cpu_count()} cpus"}


# ----------------------------------------------------------------------------- arms
def _dist_max(ms, device, world):
    if world > 1:
        t = torch.tensor([ms], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    return ms


def run_ours(args, world, rank, local):
    from flashinfer_bench_tma_thrust_b200 import decode
    from flashinfer_bench_tma_thrust_b200.partition import plan_decode
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    pk = peaks()
    hbm = pk[0]
    K, Wm = args.steps, args.warmup
    result = {"n_gpus": world, "steps": K, "warmup": Wm, "higher_is_better": True,
              "scaling": "weak", "vs_baseline": None, "data": "synthetic"}
    if args.workload == "decode_fp8":
        # the reduced-precision option alone (a separately reported figure; used for its
        # ncu summary): fp8 E4M3 state + row scales, B per GPU as the decode workload
        b0, b1 = plan_decode(args.batch * world, world)[rank]
        x, info = decode_workload(device, seed=1000 + b0, B=b1 - b0)
        sampler = ClockSampler(device)
        fp = decode_fp8_measure(x, info, K, Wm, device, world, float("nan"))
        result.update({"metric": "GDN decode fp8-state GB/s (fp8 state + row scales / step time)",
                       "value": fp["value"], "unit": "GB/s", "ms_per_step": fp["ms_per_step"],
                       "dtype": "fp8 e4m3 state, f32 math", "clocks": sampler.stop(),
                       "config": {"workload": f"gdn_decode fp8 state B={args.batch}/GPU"},
                       "gpu_launches": K, "frac_of_hbm": fp["frac_of_hbm"]})
        return result
    if args.workload == "decode":
        # the global batch (B per GPU x world) sharded by sequence with the partitioner
        B_glob = args.batch * world
        b0, b1 = plan_decode(B_glob, world)[rank]
        x, info = decode_workload(device, seed=1000 + b0, B=b1 - b0)
        holder = {"s": x.state.clone()}

        def step():
            _, ns = decode.kernel(x.q, x.k, x.v, holder["s"], x.A_log, x.a, x.dt_bias, x.b,
                                  x.scale)
            holder["s"] = ns

        sampler = ClockSampler(device)
        ms = time_steps(step, K, Wm, device, world)
        clocks = sampler.stop()
        ms_step = ms / K
        value = 2 * B_glob * HV * D * D * 4 / (ms_step * 1e-3) / 1e9
        # the launch's device time: per-launch event brackets include the events' own
        # overhead, so the smaller of that and the back-to-back step time is used
        k_ev = kernel_launch_ms(step, 50, device)
        k_ms = min(k_ev, ms_step)
        achieved = info["alg_bytes"] / (k_ms * 1e-3) / 1e9
        traffic = ncu_traffic("decode_b256")
        result.update({
            "metric": "GDN decode state GB/s (2*B*HV*D*D*4 / step time)",
            "value": round(value, 2), "unit": "GB/s", "ms_per_step": round(ms_step, 5),
            "dtype": "f32",
            "pct_of_8TBps": round(100.0 * value / world / 8000.0, 2),
            "config": {"workload": f"gdn_decode B={args.batch}/GPU, 16 q/k heads, 32 v heads, "
                                   "D=128, fp32 k-last state, bf16 q/k/v/a/b",
                       "global_batch": B_glob,
                       "parallelism": f"sequence-sharded x{world} (partition.plan_decode)",
                       "l2": "state (512 MiB in + 512 MiB out per GPU) larger than L2; no flush"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm,
                         "peak_source": f"{pk[3]} hbm_gbs", "unit": "GB/s",
                         "frac": round(achieved / hbm, 4), "traffic": traffic,
                         "alg_bytes_per_launch": info["alg_bytes"],
                         "kernel_ms": round(k_ms, 5), "kernel_ms_event_bracket": round(k_ev, 5)},
            "clocks": clocks, "gpu_launches": K,
        })
        if not args.no_e2e:
            jobs = [tuple(x.args())]
            result["e2e"] = e2e_measure(jobs, decode.kernel, device, world, min(K, 20),
                                        max(3, min(Wm, 3)),
                                        units=2 * B_glob * HV * D * D * 4, scale=1e-9,
                                        unit="GB/s")
        if world == 1 and rank == 0 and not args.no_cpu_baseline:
            # the same implementation and inputs as the reference arm, on the full batch
            # when three steps fit in about 40 s
            result["cpu_baseline"] = cpu_decode_time(decode_sample_size(3, 1, 40.0), 3, 1,
                                                     min_seconds=10.0)[0]
        if not args.no_extra:
            result["extra"] = {
                "decode_bf16_state": decode_bf16_measure(x, info, K, Wm, device, world, ms_step),
                "decode_fp8_state": decode_fp8_measure(x, info, K, Wm, device, world, ms_step)}
            for w, k, ke in (("prefill_varlen", 10, 10), ("prefill_long", 5, 4)):
                result["extra"][w] = prefill_measure(w, k, 3, device, world, rank, pk, args,
                                                     e2e_steps=ke)
            result["extra"]["decode_sweep"] = decode_sweep_measure(device, world, rank)
            if world == 1:
                result["extra"]["reference_v10_decode"] = reference_v10_measure(
                    x, info, device, ms_step)
    else:
        pm = prefill_measure(args.workload, K, Wm, device, world, rank, pk, args,
                             e2e_steps=min(K, 5))
        result.update({"metric": "GDN prefill tokens/s", "value": pm.pop("value"),
                       "unit": pm.pop("unit"), "ms_per_step": pm.pop("ms_per_step"),
                       "dtype": "f32 state, bf16 tensor-core operands",
                       "scaling": pm.pop("scaling")})
        pm.pop("steps"), pm.pop("warmup")
        result.update(pm)
    return result


def decode_sweep_measure(device, world, rank, batches=(1, 16, 64, 256, 1024, 4096)):
    """Decode batch sweep (global batch B sharded by sequence over the ranks with
    partition.plan_decode): per B, one CUDA graph of R decode steps, each on its own
    state buffer (R chosen so that the states of one replay exceed the L2 twice over;
    R = 1 once one state does), timed with CUDA events over whole replays; max over
    ranks. Graph replay removes the per-launch host cost that dominates B = 1 and 16."""
    from flashinfer_bench_tma_thrust_b200 import decode, workloads as W
    from flashinfer_bench_tma_thrust_b200.partition import plan_decode
    per_seq = HV * D * D * 4
    out = []
    for B in batches:
        b0, b1 = plan_decode(B, world)[rank]
        Bl = b1 - b0
        Bmax = max(e - s for s, e in plan_decode(B, world))
        # (Bl = 0: fewer sequences than ranks; this rank idles but joins the max)
        R = max(1, -(-(2 * 126 * 2 ** 20) // (max(Bl, 1) * per_seq)))
        reps = max(3, min(200, int(2e8 // (R * max(Bmax, 1) * per_seq * 2) + 1)))
        ms = 0.0
        if Bl > 0:
            xs = [W.decode_inputs(Bl, seed=7000 + 31 * b0 + r, gen_device=device, device=device)
                  for r in range(R)]
            for x in xs:  # warm up outside the capture (library load, attribute set-up)
                decode.kernel(*x.args())
            torch.cuda.synchronize(device)
            g = torch.cuda.CUDAGraph()
            keep = []
            with torch.cuda.graph(g):
                for x in xs:
                    keep.append(decode.kernel(*x.args()))
            for _ in range(3):
                g.replay()
            torch.cuda.synchronize(device)
        if world > 1:
            torch.distributed.barrier()
        if Bl > 0:
            s = torch.cuda.Event(enable_timing=True)
            e = torch.cuda.Event(enable_timing=True)
            s.record()
            for _ in range(reps):
                g.replay()
            e.record()
            e.synchronize()
            ms = s.elapsed_time(e) / (reps * R)  # per step
        ms = _dist_max(ms, device, world)
        us_step = 1000.0 * ms
        out.append({"B": B, "B_per_gpu_max": Bmax, "us_per_step": round(us_step, 2),
                    "state_gbs": round(2 * B * per_seq / (us_step * 1e-6) / 1e9, 1),
                    "buffers_rotated": R})
        if Bl > 0:
            del g, keep, xs
        torch.cuda.empty_cache()
    return out


def reference_v10_measure(x, info, device, our_ms_step, iters=50):
    """Same-box comparator: the reference's own CUDA decode kernels ("v10", cute and tma
    launchers of gdn/kernels/cute_cpp/gdn_decode_v10.cuh, built into oracle/_ref/) on
    this run's B=256, 16/32-head inputs, for each BLOCK_V its launcher supports; the
    state is ping-ponged between two buffers (a decode loop), CUDA events over `iters`
    launches. Each launched configuration's first step is checked against ours."""
    from oracle import ref_v10
    from flashinfer_bench_tma_thrust_b200 import decode
    if not ref_v10.available():
        return {"unavailable": "oracle/_ref/libref_v10.so not built (no reference checkout)"}
    B = info["B"]
    out_ref, ns_ref = decode.kernel(*x.args())
    rows = []
    for variant, vname in ((0, "cute"), (1, "tma")):
        for bv in (16, 32, 64):
            o = torch.empty(B, HV, D, dtype=torch.bfloat16, device=device)
            bufs = [x.state.clone(), torch.empty_like(x.state)]
            rc = ref_v10.decode(x.q, x.k, x.v, bufs[0], x.A_log, x.a, x.dt_bias, x.b, o, bufs[1],
                                x.scale, bv, variant)
            torch.cuda.synchronize(device)
            rec = {"launcher": vname, "BLOCK_V": bv, "launch_status": rc}
            if rc == 0:
                rec["max_abs_out_vs_ours"] = (o.float() - out_ref[:, 0].float()).abs().max().item()
                rec["max_abs_state_vs_ours"] = (bufs[1] - ns_ref).abs().max().item()
                for i in range(5):
                    ref_v10.decode(x.q, x.k, x.v, bufs[i & 1], x.A_log, x.a, x.dt_bias, x.b, o,
                                   bufs[(i + 1) & 1], x.scale, bv, variant)
                torch.cuda.synchronize(device)
                s = torch.cuda.Event(enable_timing=True)
                e = torch.cuda.Event(enable_timing=True)
                s.record()
                for i in range(iters):
                    ref_v10.decode(x.q, x.k, x.v, bufs[i & 1], x.A_log, x.a, x.dt_bias, x.b, o,
                                   bufs[(i + 1) & 1], x.scale, bv, variant)
                e.record()
                e.synchronize()
                ms = s.elapsed_time(e) / iters
                rec.update({"ms_per_step": round(ms, 5),
                            "state_gbs": round(info["state_bytes"] / (ms * 1e-3) / 1e9, 1)})
            else:
                rec["note"] = ("launch rejected: the launcher requests more dynamic shared "
                               "memory than the 48 KB default without the opt-in attribute")
            rows.append(rec)
            del bufs
    ok = [r for r in rows if r.get("ms_per_step")]
    best = min(ok, key=lambda r: r["ms_per_step"]) if ok else None
    return {"config": f"B={B}, 16 q/k heads, 32 v heads (this run's decode inputs)",
            "runs": rows,
            "best": {k: best[k] for k in ("launcher", "BLOCK_V", "state_gbs")} if best else None,
            "ours_over_best": round(best["ms_per_step"] / our_ms_step, 3) if best else None}


def decode_bf16_measure(x, info, K, Wm, device, world, fp32_ms_step):
    """Reduced-precision option, reported separately: the same decode loop with a bf16
    state (half the state bytes). value = bf16 state bytes moved per second."""
    from flashinfer_bench_tma_thrust_b200 import decode
    holder = {"s": x.state.to(torch.bfloat16)}

    def step():
        _, ns = decode.kernel_bf16_state(x.q, x.k, x.v, holder["s"], x.A_log, x.a, x.dt_bias,
                                         x.b, x.scale)
        holder["s"] = ns

    ms = time_steps(step, K, Wm, device, world)
    ms_step = ms / K
    b16 = info["state_bytes"] // 2
    hbm = peaks()[0]
    v = world * b16 / (ms_step * 1e-3) / 1e9
    return {"value": round(v, 2), "unit": "GB/s (bf16 state)",
            "ms_per_step": round(ms_step, 5), "frac_of_hbm": round(v / world / hbm, 4),
            "speedup_vs_fp32_state": round(fp32_ms_step / ms_step, 3),
            "error": "separately reported: see tests/test_decode_bf16_state_gpu.py"}


def decode_fp8_measure(x, info, K, Wm, device, world, fp32_ms_step):
    """Reduced-precision option, reported separately: FP8 E4M3 state + per-row fp32
    scales (132 bytes per 128-element row). value = fp8 state bytes moved per second."""
    from flashinfer_bench_tma_thrust_b200 import decode
    codes, sc = decode.quantize_state_fp8(x.state)
    holder = {"c": codes, "s": sc}

    def step():
        _, c, s = decode.kernel_fp8_state(x.q, x.k, x.v, holder["c"], holder["s"], x.A_log, x.a,
                                          x.dt_bias, x.b, x.scale)
        holder["c"], holder["s"] = c, s

    ms = time_steps(step, K, Wm, device, world)
    ms_step = ms / K
    b8 = info["state_bytes"] // 4 + info["state_bytes"] // (4 * 128)
    hbm = peaks()[0]
    v = world * b8 / (ms_step * 1e-3) / 1e9
    return {"value": round(v, 2),
            "unit": "GB/s (fp8 state + row scales)", "ms_per_step": round(ms_step, 5),
            "frac_of_hbm": round(v / world / hbm, 4),
            "speedup_vs_fp32_state": round(fp32_ms_step / ms_step, 3),
            "error": "separately reported: see tests/test_decode_fp8_state_gpu.py"}


PREFILL_FLOP_PER_TOKEN_HEAD = 6 * D * D + 10 * 64 * D + (2 * 64 * 64) // 3


def prefill_plan(workload, world):
    """Global sequence set of a prefill configuration and its plan over `world` ranks:
    varlen = the configuration's 8 sequences (strong scaling: (sequence, head-group)
    units spread over the ranks); long = 4 sequences of 32768 tokens per GPU (weak
    scaling: whole sequences)."""
    from flashinfer_bench_tma_thrust_b200.partition import plan_prefill
    lengths, with_state = prefill_lengths(workload)
    scaling = "strong" if workload == "prefill_varlen" else "weak"
    if workload == "prefill_long":
        lengths = lengths * world
    return lengths, with_state, scaling, plan_prefill(lengths, world, HQ, HV)


def prefill_measure(workload, K, Wm, device, world, rank, pk, args, e2e_steps=3):
    """Time K prefill steps of `workload`: this rank's calls of prefill.kernel on its
    part of the global sequence set (partition.plan_prefill / build_local_prefill); the
    step time is the max over ranks and value = global tokens / step time."""
    from flashinfer_bench_tma_thrust_b200 import prefill, workloads as W
    from flashinfer_bench_tma_thrust_b200.partition import build_local_prefill
    hbm, bf16_burst = pk[0], pk[1]
    lengths, with_state, scaling, plan = prefill_plan(workload, world)
    T_glob = sum(lengths)
    x = W.prefill_inputs(lengths, seed=2000, gen_device=device, device=device,
                         with_state=with_state)
    local = build_local_prefill(plan, rank, *x.args(), device=device)
    del x
    torch.cuda.empty_cache()
    jobs = [c[4] for c in local.calls]
    T_loc = sum(sum(c[3]) for c in local.calls)
    flops = sum(sum(c[3]) * (c[1] - c[0]) for c in local.calls) * PREFILL_FLOP_PER_TOKEN_HEAD

    def nbytes(t):
        return t.numel() * t.element_size() if isinstance(t, torch.Tensor) else 0
    # compulsory HBM bytes: every input once (q, k, v, gates, cu_seqlens, initial state),
    # outputs and final states written once
    comp_bytes = 0
    for (h0, h1, seqs, lens, a) in local.calls:
        comp_bytes += sum(nbytes(t) for t in a) + sum(lens) * (h1 - h0) * D * 2 + \
            len(seqs) * (h1 - h0) * D * D * 4
    launches = sum(prefill.launches_per_call(len(c[2]), sum(c[3]), c[1] - c[0])
                   for c in local.calls)

    def step():
        for a in jobs:
            prefill.kernel(*a)

    sampler = ClockSampler(device)
    ms = time_steps(step, K, Wm, device, world)
    clocks = sampler.stop()
    ms_step = ms / K
    k_ms = kernel_launch_ms(step, 3, device) if jobs else 0.0
    k_ms = min(k_ms, ms_step) if jobs else 0.0
    achieved = flops / (k_ms * 1e-3) / 1e12 if k_ms else 0.0
    dram = comp_bytes / (k_ms * 1e-3) / 1e9 if k_ms else 0.0
    roof = {"bound": "tensor", "achieved": round(achieved, 2), "peak": bf16_burst,
            "peak_source": f"{pk[3]} bf16_tflops (burst: the call is timed alone)",
            "unit": "TFLOP/s", "frac": round(achieved / bf16_burst, 4),
            "traffic": ncu_traffic(workload) if world == 1 else None,
            "flop_per_token": HV * PREFILL_FLOP_PER_TOKEN_HEAD, "call_ms": round(k_ms, 4),
            "dram": {"compulsory_bytes": comp_bytes, "achieved_gbs": round(dram, 1),
                     "peak": hbm, "frac": round(dram / hbm, 4)}}
    out = {"value": round(T_glob / (ms_step * 1e-3), 1), "unit": "tokens/s",
           "ms_per_step": round(ms_step, 4), "steps": K, "warmup": Wm, "scaling": scaling,
           "config": {"workload": f"gdn_prefill {workload}: lengths {lengths[:8]}"
                                  f"{'...' if len(lengths) > 8 else ''} (T={T_glob} total), "
                                  "16 q/k heads, 32 v heads, D=128, chunk 64, "
                                  f"{'initial state N(0,0.02)' if with_state else 'zero state'}",
                      "global_tokens": T_glob, "tokens_this_rank": T_loc,
                      "parallelism": f"partition.plan_prefill x{world}: {plan.groups} head "
                                     f"group(s) per sequence",
                      "l2": "inputs (q/k/v >= 100 MB) larger than L2; no flush"},
           "roofline": roof, "clocks": clocks, "gpu_launches": K * launches}
    if not args.no_e2e and jobs is not None:
        out["e2e"] = e2e_measure(jobs, prefill.kernel, device, world, e2e_steps, 4,
                                 units=T_glob, scale=1.0, unit="tokens/s")
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_prefill_time(lengths, with_state, 3, 1, min_seconds=10.0)
    return out


def e2e_measure(jobs, fn, device, world, K, Wm, units, scale, unit):
    """The metric through the public API (`fn` = decode.kernel / prefill.kernel) with
    host buffers: every step copies all inputs of this rank's calls (`jobs`, tuples of
    kernel arguments) from pinned host memory, runs the calls, and reads every output
    (o and new_state) back into pinned host memory. Copies run on their own streams with
    two buffer sets, so step i's device->host copy overlaps step i+1's host->device copy
    and the kernels (the two PCIe directions work concurrently); the timed region spans
    all streams; max over ranks. value = units per step / step time x scale."""
    host_sets, dev_sets, outs_h = [], [], []
    probe = [fn(*a) for a in jobs]
    for j in range(2):
        host_sets.append([[t.cpu().pin_memory() if isinstance(t, torch.Tensor) else t
                           for t in a] for a in jobs])
        dev_sets.append([[torch.empty_like(t, device=device) if isinstance(t, torch.Tensor)
                          else t for t in a] for a in jobs])
        outs_h.append([[torch.empty(o.shape, dtype=o.dtype).pin_memory() for o in res]
                       for res in probe])
    del probe
    h2d = sum(t.numel() * t.element_size() for a in host_sets[0] for t in a
              if isinstance(t, torch.Tensor))
    d2h = sum(o.numel() * o.element_size() for res in outs_h[0] for o in res)
    comp = torch.cuda.current_stream(device)
    s_in = torch.cuda.Stream(device)
    s_out = torch.cuda.Stream(device)
    free = [torch.cuda.Event() for _ in range(2)]   # set j's device inputs consumed
    ready = [torch.cuda.Event() for _ in range(2)]  # set j's inputs on the device
    done = [torch.cuda.Event() for _ in range(2)]   # step on set j computed
    drained = [torch.cuda.Event() for _ in range(2)]  # set j's results on the host
    for j in range(2):
        free[j].record(comp)
        drained[j].record(s_out)
    it = [0]
    held = [None, None]  # each set's last results, kept until their copy-out is done

    def step():
        j = it[0] % 2
        it[0] += 1
        if held[j] is not None:
            # the results of two steps ago leave the host's hands only once copied out,
            # so the allocator can reuse their memory without a stream-use record
            drained[j].synchronize()
            held[j] = None
        with torch.cuda.stream(s_in):
            s_in.wait_event(free[j])
            for dst_a, src_a in zip(dev_sets[j], host_sets[j]):
                for dst, src in zip(dst_a, src_a):
                    if isinstance(src, torch.Tensor):
                        dst.copy_(src, non_blocking=True)
            ready[j].record(s_in)
        comp.wait_event(ready[j])
        comp.wait_event(drained[j])  # host buffers of set j free again
        results = [fn(*a) for a in dev_sets[j]]
        free[j].record(comp)
        done[j].record(comp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(done[j])
            for res, res_h in zip(results, outs_h[j]):
                for o, oh in zip(res, res_h):
                    oh.copy_(o, non_blocking=True)
            drained[j].record(s_out)
        held[j] = results

    for _ in range(Wm):
        step()
    torch.cuda.synchronize(device)
    if world > 1:
        torch.distributed.barrier()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(comp)
    s_in.wait_stream(comp)
    s_out.wait_stream(comp)
    for _ in range(K):
        step()
    comp.wait_stream(s_in)
    comp.wait_stream(s_out)
    end.record(comp)
    end.synchronize()
    torch.cuda.synchronize(device)
    ms = _dist_max(start.elapsed_time(end), device, world)
    last = outs_h[(K + Wm - 1) % 2]
    ok = all(bool(o.float().isfinite().all()) for res in last for o in res)
    return {"value": round(units / (ms / K * 1e-3) * scale, 3), "unit": unit,
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": K,
            "ms_per_step": round(ms / K, 3),
            "overlap": "copies on separate streams, 2 buffer sets", "outputs_finite": ok}


def run_reference(args):
    """Reference arm: the reference's own CPU implementation of the path (its PyTorch
    baseline, or the oracle's restatement of it where that file is not staged), on the
    host cores with all threads, on the same configuration as our arm."""
    K, Wm = args.steps, args.warmup
    if args.workload == "decode":
        B_sample = decode_sample_size(K, Wm)
        # guard against a cost that grows faster than the batch (host memory pressure)
        while B_sample > 1 and cpu_decode_time(B_sample, 1, 0)[1] * (K + Wm) > 225.0:
            B_sample //= 2
        cb, per = cpu_decode_time(B_sample, K, Wm)
        metric = "GDN decode state GB/s (2*B*HV*D*D*4 / step time)"
        cfg = {"workload": f"gdn_decode B={args.batch}/GPU, 16 q/k heads, 32 v heads, D=128, "
                           "fp32 k-last state, bf16 q/k/v/a/b",
               "global_batch": args.batch * args.gpus, "cpu_batch_per_step": B_sample,
               "same_config": B_sample == args.batch}
        ms_step = per * 1e3
    else:
        lengths, with_state = prefill_lengths(args.workload)
        cb = cpu_prefill_time(lengths, with_state, K, Wm, tokens_per_seq=16)
        metric = "GDN prefill tokens/s"
        cfg = {"workload": f"gdn_prefill {args.workload}: lengths {lengths[:8]}, 16 q/k heads, "
                           "32 v heads", "same_config": False}
        ms_step = None
    value = cb["value"]
    line = {"impl": "reference", "metric": metric, "value": round(value, 4), "unit": cb["unit"],
            "n_gpus": args.gpus, "steps": K, "warmup": Wm,
            "ms_per_step": round(ms_step, 3) if ms_step else None,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": cfg,
            "cpu_baseline": {"value": round(value, 4), "unit": cb["unit"], "cores": cb["cores"],
                             "kind": cb["kind"], "sample": cb["sample"]},
            "e2e": {"value": round(value, 4), "unit": cb["unit"], "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
            "gpu_launches": 0}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawTextHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="decode",
                    choices=["decode", "decode_fp8", "prefill_varlen", "prefill_long"])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=256, help="decode sequences per GPU")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra", action="store_true",
                    help="decode run only: skip the prefill configurations in 'extra'")
    args = ap.parse_args()
    if args.steps is None:
        args.steps = 2000 if args.workload == "decode" else 20
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    world, rank, local = dist_env()
    if args.impl == "reference":
        if rank == 0:
            run_reference(args)
        return
    if world > 1:
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", device_id=torch.device("cuda", local))
    try:
        res = run_ours(args, world, rank, local)
        if rank == 0:
            line = {"metric": res.pop("metric"), "value": res.pop("value"), "unit": res.pop("unit")}
            line.update(res)
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
