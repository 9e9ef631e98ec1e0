"""Benchmark of the GDN hot path on B200 — prints ONE JSON line (rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload decode|prefill_varlen|prefill_long]
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
  initial state ~N(0,0.02). Metric: tokens/s.
* ``prefill_long``: 4 sequences x 32768 tokens per GPU, zero initial state. Metric: tokens/s.

Multi-GPU (torchrun, one process per GPU): every rank owns its own batch slice
(weak scaling, no data-path collective); the step time is the max over ranks.

``--impl reference`` times the reference's CPU implementation of the same path
(the oracle restatement of the reference's PyTorch baseline, run on the host
cores with all threads) on a bounded sample of the workload per step.
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


def cpu_decode_baseline(seconds=10.0, sample_B=16):
    """Oracle (restated reference PyTorch decode) on the host cores, on a sample of the
    B=256 workload's sequences per step."""
    from flashinfer_bench_tma_thrust_b200 import workloads as W
    from oracle import gdn_oracle
    x = W.decode_inputs(256, seed=0)
    sl = [t[:sample_B] if isinstance(t, torch.Tensor) and t.dim() > 1 else t for t in x.args()]
    gdn_oracle.decode(*sl)  # warm-up
    n, t0 = 0, time.perf_counter()
    while True:
        gdn_oracle.decode(*sl)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds and n >= 3:
            break
    sb = 2 * sample_B * HV * D * D * 4
    return {"value": sb * n / el / 1e9, "unit": "GB/s", "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": f"{sample_B} of the 256 sequences per step, {n} steps in {el:.1f} s, "
                      f"torch CPU fp32, {torch.get_num_threads()} threads of "
                      f"{os.cpu_count()} cpus"}


def cpu_prefill_baseline(lengths, seconds=10.0, tokens_per_seq=64):
    from flashinfer_bench_tma_thrust_b200 import workloads as W
    from oracle import gdn_oracle
    sub = [min(l, tokens_per_seq) for l in lengths]
    x = W.prefill_inputs(sub, seed=0)
    n, t0 = 0, time.perf_counter()
    while True:
        gdn_oracle.prefill(*x.args())
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds and n >= 1:
            break
    return {"value": sum(sub) * n / el, "unit": "tokens/s", "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": f"first {tokens_per_seq} tokens of each of the {len(lengths)} sequences "
                      f"({sum(sub)} tokens) per step, {n} steps in {el:.1f} s, torch CPU fp32, "
                      f"{torch.get_num_threads()} threads of {os.cpu_count()} cpus"}


# ----------------------------------------------------------------------------- arms
def run_ours(args, world, rank, local):
    from flashinfer_bench_tma_thrust_b200 import decode, prefill
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    hbm, bf16, bf16_sus, peak_src = peaks()
    K, Wm = args.steps, args.warmup
    result = {"n_gpus": world, "steps": K, "warmup": Wm, "higher_is_better": True,
              "scaling": "weak", "vs_baseline": None, "data": "synthetic"}
    if args.workload == "decode":
        x, info = decode_workload(device, seed=1000 + rank, B=args.batch)
        B = info["B"]
        holder = {"s": x.state.clone()}

        def step():
            _, ns = decode.kernel(x.q, x.k, x.v, holder["s"], x.A_log, x.a, x.dt_bias, x.b,
                                  x.scale)
            holder["s"] = ns

        sampler = ClockSampler(device)
        ms = time_steps(step, K, Wm, device, world)
        clocks = sampler.stop()
        ms_step = ms / K
        value = world * info["state_bytes"] / (ms_step * 1e-3) / 1e9
        k_ms = kernel_launch_ms(step, 50, device)
        achieved = info["alg_bytes"] / (k_ms * 1e-3) / 1e9
        traffic = ncu_traffic("decode_b256")
        result.update({
            "metric": "GDN decode state GB/s (2*B*HV*D*D*4 / step time)",
            "value": round(value, 2), "unit": "GB/s", "ms_per_step": round(ms_step, 5),
            "dtype": "f32",
            "pct_of_8TBps": round(100.0 * value / world / 8000.0, 2),
            "config": {"workload": f"gdn_decode B={B}/GPU, 16 q/k heads, 32 v heads, D=128, "
                                   "fp32 k-last state, bf16 q/k/v/a/b",
                       "global_batch": B * world, "parallelism": f"sequence-sharded x{world}",
                       "l2": "state (512 MiB in + 512 MiB out per GPU) larger than L2; no flush"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm,
                         "peak_source": peak_src, "unit": "GB/s",
                         "frac": round(achieved / hbm, 4), "traffic": traffic,
                         "alg_bytes_per_launch": info["alg_bytes"],
                         "kernel_ms": round(k_ms, 5)},
            "clocks": clocks, "gpu_launches": K,
        })
        if not args.no_e2e:
            result["e2e"] = decode_e2e(x, info, device, world, min(K, 20), max(3, min(Wm, 3)))
        if world == 1 and rank == 0 and not args.no_cpu_baseline:
            result["cpu_baseline"] = cpu_decode_baseline()
    else:
        pm = prefill_measure(args.workload, K, Wm, device, world, rank, peak=bf16_sus,
                             peak_src=peak_src)
        lengths, T = pm.pop("lengths"), pm.pop("T")
        result.update({
            "metric": "GDN prefill tokens/s", "value": pm["value"], "unit": "tokens/s",
            "ms_per_step": pm["ms_per_step"], "dtype": "f32 state, bf16 tensor-core operands",
            "config": {"workload": f"gdn_prefill {args.workload}: lengths {lengths[:8]}"
                                   f"{'...' if len(lengths) > 8 else ''} (T={T}/GPU), 16 q/k "
                                   "heads, 32 v heads, D=128, chunk 64",
                       "global_tokens": T * world, "parallelism": f"sequence-sharded x{world}",
                       "l2": "inputs (q/k/v >= 100 MB per GPU) larger than L2; no flush"},
            "roofline": pm["roofline"], "clocks": pm["clocks"],
            "gpu_launches": K * prefill.launches_per_call(len(lengths), T, 32),
        })
        if world == 1 and rank == 0 and not args.no_cpu_baseline:
            result["cpu_baseline"] = cpu_prefill_baseline(lengths)
    if args.workload == "decode" and not args.no_extra:
        result["extra"] = {"decode_bf16_state": decode_bf16_measure(x, info, K, Wm, device,
                                                                    world, ms_step),
                           "decode_fp8_state": decode_fp8_measure(x, info, K, Wm, device,
                                                                  world, ms_step)}
        result["extra"].update({
            w: prefill_measure(w, k, 3, device, world, rank, peak=bf16_sus, peak_src=peak_src,
                               brief=True)
            for w, k in (("prefill_varlen", 10), ("prefill_long", 5))})
        result["extra"]["decode_sweep"] = decode_sweep_measure(device, world, rank)
    return result


def decode_sweep_measure(device, world, rank, batches=(1, 16, 64, 256, 1024, 4096)):
    """Decode batch sweep (global batch B sharded by sequence over the ranks): per B, one
    CUDA graph of R decode steps, each on its own state buffer (R chosen so that the
    states of one replay exceed the L2 twice over; R = 1 once one state does), timed
    with CUDA events over whole replays; max over ranks. Graph replay removes the
    per-launch host cost that dominates B = 1 and 16."""
    from flashinfer_bench_tma_thrust_b200 import decode, workloads as W
    per_seq = HV * D * D * 4
    out = []
    for B in batches:
        Bl = -(-B // world)
        R = max(1, -(-(2 * 126 * 2 ** 20) // (Bl * per_seq)))
        xs = [W.decode_inputs(Bl, seed=7000 + 31 * rank + r, gen_device=device, device=device)
              for r in range(R)]
        for x in xs:  # warm up outside the capture (library load, attribute set-up)
            decode.kernel(*x.args())
        torch.cuda.synchronize(device)
        g = torch.cuda.CUDAGraph()
        keep = []
        with torch.cuda.graph(g):
            for x in xs:
                keep.append(decode.kernel(*x.args()))
        reps = max(3, min(200, int(2e8 // (R * Bl * per_seq * 2) + 1)))
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize(device)
        if world > 1:
            torch.distributed.barrier()
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(reps):
            g.replay()
        e.record()
        e.synchronize()
        ms = s.elapsed_time(e)
        if world > 1:
            t = torch.tensor([ms], device=device)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            ms = float(t.item())
        us_step = 1000.0 * ms / (reps * R)
        out.append({"B": B, "B_per_gpu": Bl, "us_per_step": round(us_step, 2),
                    "state_gbs": round(world * 2 * Bl * per_seq / (us_step * 1e-6) / 1e9, 1),
                    "buffers_rotated": R})
        del g, keep, xs
        torch.cuda.empty_cache()
    return out


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
    return {"value": round(world * b16 / (ms_step * 1e-3) / 1e9, 2), "unit": "GB/s (bf16 state)",
            "ms_per_step": round(ms_step, 5),
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
    return {"value": round(world * b8 / (ms_step * 1e-3) / 1e9, 2),
            "unit": "GB/s (fp8 state + row scales)", "ms_per_step": round(ms_step, 5),
            "speedup_vs_fp32_state": round(fp32_ms_step / ms_step, 3),
            "error": "separately reported: see tests/test_decode_fp8_state_gpu.py"}


def prefill_measure(workload, K, Wm, device, world, rank, peak, peak_src, brief=False):
    """Time K prefill steps (one prefill.kernel call each) of `workload` on this rank."""
    from flashinfer_bench_tma_thrust_b200 import prefill, workloads as W
    lengths, with_state = prefill_lengths(workload)
    x = W.prefill_inputs(lengths, seed=2000 + rank, gen_device=device, device=device,
                         with_state=with_state)
    T = sum(lengths)

    def step():
        prefill.kernel(*x.args())

    sampler = ClockSampler(device)
    ms = time_steps(step, K, Wm, device, world)
    clocks = sampler.stop()
    ms_step = ms / K
    flop_per_token = HV * (6 * D * D + 10 * 64 * D + (2 * 64 * 64) // 3)
    k_ms = kernel_launch_ms(step, 3, device)
    achieved = T * flop_per_token / (k_ms * 1e-3) / 1e12
    roof = {"bound": "tensor", "achieved": round(achieved, 2), "peak": peak,
            "peak_source": peak_src + " (sustained bf16)", "unit": "TFLOP/s",
            "frac": round(achieved / peak, 4), "traffic": ncu_traffic(workload),
            "flop_per_token": flop_per_token, "call_ms": round(k_ms, 4)}
    out = {"value": round(world * T / (ms_step * 1e-3), 1), "unit": "tokens/s",
           "ms_per_step": round(ms_step, 4), "steps": K, "warmup": Wm, "roofline": roof}
    if brief:
        out["tokens_per_gpu"] = T
        return out
    out.update({"lengths": lengths, "T": T, "clocks": clocks})
    return out


def decode_e2e(x, info, device, world, K, Wm):
    """Same metric through the public API (decode.kernel) with host buffers: every step
    copies its inputs from pinned host memory and reads the output and the new state
    back into pinned host memory. Copies run on their own streams with two buffer sets,
    so step i's device->host copy overlaps step i+1's host->device copy and the kernel
    (the two PCIe directions work concurrently); the timed region spans all streams."""
    from flashinfer_bench_tma_thrust_b200 import decode
    B = info["B"]
    host_sets, dev_sets, out_h, ns_h = [], [], [], []
    for j in range(2):
        host_sets.append([t.cpu().pin_memory() if isinstance(t, torch.Tensor) else t
                          for t in x.args()])
        dev_sets.append([torch.empty_like(t, device=device) if isinstance(t, torch.Tensor) else t
                         for t in x.args()])
        out_h.append(torch.empty(B, 1, HV, D, dtype=torch.bfloat16).pin_memory())
        ns_h.append(torch.empty(B, HV, D, D, dtype=torch.float32).pin_memory())
    h2d = sum(t.numel() * t.element_size() for t in host_sets[0] if isinstance(t, torch.Tensor))
    d2h = out_h[0].numel() * 2 + ns_h[0].numel() * 4
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

    def step():
        j = it[0] % 2
        it[0] += 1
        with torch.cuda.stream(s_in):
            s_in.wait_event(free[j])
            for dst, src in zip(dev_sets[j], host_sets[j]):
                if isinstance(src, torch.Tensor):
                    dst.copy_(src, non_blocking=True)
            ready[j].record(s_in)
        comp.wait_event(ready[j])
        comp.wait_event(drained[j])  # host buffers of set j free again
        out, ns = decode.kernel(*dev_sets[j])
        free[j].record(comp)
        done[j].record(comp)
        out.record_stream(s_out)
        ns.record_stream(s_out)
        with torch.cuda.stream(s_out):
            s_out.wait_event(done[j])
            out_h[j].copy_(out, non_blocking=True)
            ns_h[j].copy_(ns, non_blocking=True)
            drained[j].record(s_out)

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
    ms = start.elapsed_time(end)
    if world > 1:
        t = torch.tensor([ms], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    # the results of the last step really arrived: compare with a synchronous call
    ok = torch.equal(out_h[(K + Wm - 1) % 2].float().isfinite().all().reshape(1),
                     torch.ones(1, dtype=torch.bool))
    return {"value": round(world * info["state_bytes"] / (ms / K * 1e-3) / 1e9, 3),
            "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": K,
            "ms_per_step": round(ms / K, 3), "overlap": "copies on separate streams, 2 buffer sets",
            "outputs_finite": bool(ok)}


def run_reference(args):
    """Reference arm: the reference's PyTorch path (restated in oracle/) on the host CPU."""
    from flashinfer_bench_tma_thrust_b200 import workloads as W
    from oracle import gdn_oracle
    torch.set_num_threads(os.cpu_count() or 1)
    K, Wm = args.steps, args.warmup
    if args.workload == "decode":
        sample_B = 4
        x = W.decode_inputs(256, seed=1000)
        sl = [t[:sample_B] if isinstance(t, torch.Tensor) and t.dim() > 1 else t
              for t in x.args()]
        fn = lambda: gdn_oracle.decode(*sl)  # noqa: E731
        units = 2 * sample_B * HV * D * D * 4
        metric, unit = "GDN decode state GB/s (2*B*HV*D*D*4 / step time)", "GB/s"
        scale = 1e-9
        sample = f"{sample_B} of the 256 sequences of the decode workload per step"
        cfg = "gdn_decode B=256/GPU, 16 q/k heads, 32 v heads, D=128, fp32 k-last state"
    else:
        lengths, with_state = prefill_lengths(args.workload)
        sub = [min(l, 16) for l in lengths]
        x = W.prefill_inputs(sub, seed=2000, with_state=with_state)
        fn = lambda: gdn_oracle.prefill(*x.args())  # noqa: E731
        units = sum(sub)
        metric, unit, scale = "GDN prefill tokens/s", "tokens/s", 1.0
        sample = f"first 16 tokens of each of the {len(lengths)} sequences per step"
        cfg = f"gdn_prefill {args.workload}: lengths {lengths[:8]}, 16 q/k heads, 32 v heads"
    for _ in range(Wm):
        fn()
    t0 = time.perf_counter()
    for _ in range(K):
        fn()
    el = time.perf_counter() - t0
    value = units * K / el * scale
    cores = torch.get_num_threads()
    line = {"impl": "reference", "metric": metric, "value": round(value, 4), "unit": unit,
            "n_gpus": args.gpus, "steps": K, "warmup": Wm, "ms_per_step": round(el / K * 1e3, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": {"workload": cfg},
            "cpu_baseline": {"value": round(value, 4), "unit": unit, "cores": cores,
                             "kind": "port",
                             "sample": f"{sample}; torch CPU fp32 restatement of the reference "
                                       f"PyTorch baseline, {cores} threads"},
            "e2e": {"value": round(value, 4), "unit": unit, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
            "gpu_launches": 0}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawTextHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="decode",
                    choices=["decode", "prefill_varlen", "prefill_long"])
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
