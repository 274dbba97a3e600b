#!/usr/bin/env python
"""Benchmark of the fused RMSNorm -> Linear hot path (Kimi K2.6 kv_b shape).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step is one fused RMSNorm -> Linear call over one 512-token batch of the
kimi_kv_b workload (x [512, 512] bf16, W_fused [16384, 512], out [512, 16384]).
Steps rotate over enough (x, W, out) buffer sets that the working set is
about twice the 126 MB L2, so every call streams W and out from/to HBM.  The
K timed steps are captured as one CUDA graph (one node per call) and replayed,
bracketed by a barrier and torch.cuda.synchronize() on both sides, timed with
CUDA events on the launching stream.  That K-step window is repeated (at least 5 times and
until about 200 ms have been timed); each window's time is the max over ranks
and the reported time is the median window.  With N > 1 (torchrun, one rank
per GPU) each rank processes its own 512-token shard with its own weight
replica and there is no collective on the data path (weak scaling).

Besides the headline, the JSON line carries the token-partitioned
configurations at this N: ``long_prefill`` (q_b and kv_b at 4096 tokens in
total, 4096/N rows per rank, strong scaling) and ``int8_stack`` (61 layers of
int8 q_b + int8 kv_b at 2048 tokens in total, 2048/N rows per rank).

One JSON line is printed by rank 0.  ``--profile CASE`` instead runs one case's
kernel a few times with no timing, for ncu captures.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import re
import statistics
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PROJECT = os.path.join(REPO, "kimi26-h100-rmsnorm-swiglu-fusion_b200")
for _p in (PROJECT, REPO):
    if _p not in sys.path:
        sys.path.insert(0, _p)

EPS = 1e-5
L2_BYTES = 126 * 1024 * 1024
HEADLINE = "kimi_kv_b"
# name -> (tokens M, hidden K, out N)
SHAPES = {
    "kimi_q_b": (512, 1536, 12288),
    "kimi_kv_b": (512, 512, 16384),
    "kimi_q_b_long": (4096, 1536, 12288),
    "kimi_kv_b_long": (4096, 512, 16384),
    "decode_m1": (1, 4096, 6144),
    "decode_m8": (8, 4096, 6144),
    "decode_m32": (32, 4096, 6144),
    "decode_m128": (128, 4096, 6144),
}
METRIC = "fused RMSNorm+Linear TFLOP/s at the Kimi kv_b shape (512x512 -> 16384, bf16)"
NVML_REASONS = {
    0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
    0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
    0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
}


# Cases --profile can run (one kernel, a few launches, no timing): the linear
# shapes above plus the int8, SwiGLU and GQA workloads of the sweep.
PROFILE_CASES = sorted(list(SHAPES) + ["int8_q_b", "int8_q_b_256", "int8_kv_b_256",
                                       "int8_layer_256",
                                       "swiglu_prefill", "swiglu_decode_m8",
                                       "gqa_decode_llama"])
# Token-partitioned configurations: (total tokens, hidden, out).
LONG_PREFILL = {"kimi_q_b_long": (4096, 1536, 12288), "kimi_kv_b_long": (4096, 512, 16384)}
STACK_LAYERS = 61
STACK_TOKENS = 2048
STACK_SHAPES = (("q_b", 1536, 12288), ("kv_b", 512, 16384))


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(SHAPES), default=HEADLINE)
    ap.add_argument("--no-sweep", action="store_true", help="skip the per-config sweep")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline")
    ap.add_argument("--no-partitioned", action="store_true",
                    help="skip the long_prefill and int8_stack configurations")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--min-timed-ms", type=float, default=200.0,
                    help="repeat the K-step window until this much has been timed")
    ap.add_argument("--profile", choices=PROFILE_CASES,
                    help="run CASE's kernel --steps times after --warmup calls, untimed (ncu)")
    ap.add_argument("--gqa-only", action="store_true",
                    help="time only the GQA decode-attention workload (one JSON line)")
    return ap.parse_args()


def flops_of(M, K, N):
    return 2.0 * M * K * N


def bytes_of(M, K, N, elem=2):
    return float(elem) * (M * K + N * K + M * N)


def bytes_of_w8(M, K, N):
    """x and out in bf16, int8 weight, fp32 per-channel scales."""
    return 2.0 * M * K + N * K + 4.0 * N + 2.0 * M * N


def read_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, 1590.0, "fallback"


def roofline_us(flops, nbytes, hbm_gbs, tflops_peak):
    return max(flops / (tflops_peak * 1e12), nbytes / (hbm_gbs * 1e9)) * 1e6


def read_profiled_traffic(kernel: str, workload: str):
    """Per-launch DRAM bytes recorded from an ncu capture in profiles/."""
    path = os.path.join(REPO, "profiles", f"{kernel}__{workload}.md")
    try:
        text = open(path).read()
    except OSError:
        return None
    m = re.search(r"traffic_bytes_per_launch\s*[:=]\s*([0-9.eE+]+)", text)
    return float(m.group(1)) if m else None


def make_config(name, world):
    """The workload identity, the same dict in both arms."""
    M, K, N = SHAPES[name]
    return {"workload": name, "tokens_per_gpu": M, "hidden": K, "out": N,
            "parallelism": (f"dp{world}: token-partitioned, replicated W, no collective"
                            if world > 1 else "single GPU"),
            "l2": "GPU arm: each call's (x, W, out) set rotates among sets totalling about "
                  "twice the 126 MB L2 (flushed by rotation); CPU reference arm: host memory"}


class Comm:
    """Barrier / max / gather over the ranks of one job (no-ops at one rank)."""

    def __init__(self, world, local_rank, device):
        self.world, self.local_rank, self.device = world, local_rank, device

    def barrier(self):
        if self.world > 1:
            import torch.distributed as dist

            dist.barrier(device_ids=[self.local_rank])

    def max_(self, values):
        import torch

        t = torch.tensor(values, device=self.device, dtype=torch.float64)
        if self.world > 1:
            import torch.distributed as dist

            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return [float(v) for v in t.tolist()]

    def gather(self, value):
        import torch

        t = torch.tensor([value], device=self.device, dtype=torch.float64)
        if self.world == 1:
            return [value]
        import torch.distributed as dist

        out = [torch.zeros_like(t) for _ in range(self.world)]
        dist.all_gather(out, t)
        return [float(o.item()) for o in out]


LOCAL = None  # Comm of a single rank, set in run_ours


def spread(values):
    return {"min": round(min(values), 3), "median": round(statistics.median(values), 3),
            "max": round(max(values), 3)}


# ----------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clock, power and clock-event reasons through NVML."""

    def __init__(self, torch_device_index: int, period_s: float = 0.005):
        self.samples = []
        self.period = period_s
        self._stop = threading.Event()
        self._thread = None
        self.max_mhz = None
        self.handle = None
        try:
            import pynvml
            import torch

            pynvml.nvmlInit()
            self.nv = pynvml
            props = torch.cuda.get_device_properties(torch_device_index)
            uuid = getattr(props, "uuid", None)
            h = None
            if uuid is not None:
                try:
                    h = pynvml.nvmlDeviceGetHandleByUUID(f"GPU-{uuid}")
                except Exception:
                    h = None
            if h is None:
                h = pynvml.nvmlDeviceGetHandleByIndex(torch_device_index)
            self.handle = h
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
            self._reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                getattr(pynvml, "nvmlDeviceGetCurrentClocksThrottleReasons")
        except Exception as e:  # NVML missing: report no clocks rather than guess
            self.error = str(e)

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM)
                reasons = int(self._reasons(self.handle))
                power = nv.nvmlDeviceGetPowerUsage(self.handle) / 1000.0
                self.samples.append((sm, reasons, power))
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.handle is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()
        return False

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        busy = [s for s in self.samples if not (s[1] & 0x1)] or self.samples
        reasons = 0
        for s in busy:
            reasons |= s[1]
        names = [n for bit, n in NVML_REASONS.items() if reasons & bit and bit != 0x1]
        return {"sm_mhz": statistics.median(s[0] for s in busy), "sm_max_mhz": self.max_mhz,
                "reasons": names, "samples": len(busy),
                "power_w_max": round(max(s[2] for s in busy), 1)}


# -------------------------------------------------------------- workloads
def gpu_inputs(M, K, N, seed, device):
    import torch

    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn(M, K, generator=g, device=device, dtype=torch.float32).to(torch.bfloat16)
    gamma = (1.0 + 0.1 * torch.randn(K, generator=g, device=device)).to(torch.bfloat16)
    W = (torch.randn(N, K, generator=g, device=device) / math.sqrt(K)).to(torch.bfloat16)
    return x, gamma, W


def unfused_torch(x, gamma, W, eps):
    """The reference's unfused baseline on GPU: linear(SimpleRMSNorm(x))."""
    import torch
    import torch.nn.functional as F

    variance = x.float().pow(2).mean(dim=-1, keepdim=True)
    y = x * torch.rsqrt(variance + eps).to(x.dtype) * gamma.to(x.dtype)
    return F.linear(y, W)


class Rotation:
    """S independent (x, W_fused, out) sets; S chosen so S * set_bytes >= 2 * L2."""

    def __init__(self, M, K, N, device, seed=1234, min_sets=2, w_seed=None):
        import torch

        set_bytes = bytes_of(M, K, N)
        self.S = max(min_sets, int(math.ceil(2 * L2_BYTES / set_bytes)))
        self.xs, self.gammas, self.ws, self.wf, self.outs = [], [], [], [], []
        for s in range(self.S):
            x, gamma, W = gpu_inputs(M, K, N, seed + s, device)
            if w_seed is not None:  # weights shared by every rank (replicas)
                _, gamma, W = gpu_inputs(1, K, N, w_seed + s, device)
            self.xs.append(x)
            self.gammas.append(gamma)
            self.ws.append(W)
            self.wf.append(W * gamma)
            self.outs.append(torch.empty(M, N, dtype=torch.bfloat16, device=device))
        self.set_bytes = set_bytes

    def describe(self):
        tot = self.S * self.set_bytes
        return f"rotating {self.S} (x, W, out) sets, {tot / 1e6:.0f} MB > 126 MB L2"


def time_windows(fns, steps, warmup, comm, min_total_ms=200.0, max_windows=2000):
    """Times `steps` calls fns[i % S] captured as ONE CUDA graph (one node per
    call, back to back as a serving loop issues them), as one window bracketed
    by a barrier and a synchronize on both sides (CUDA events on the launching
    stream).  The window is repeated (>= 5 times, until about `min_total_ms`
    has been timed; every rank runs the same count).  Returns (this rank's ms
    per window, max over ranks per window)."""
    import torch

    S = len(fns)
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        for f in fns:  # eager warm call: attributes, tensor-map entry point
            f()
    torch.cuda.current_stream().wait_stream(stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for i in range(steps):
            fns[i % S]()
    for _ in range(max(1, math.ceil(warmup / steps))):
        graph.replay()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)

    def window():
        comm.barrier()
        torch.cuda.synchronize()
        start.record()
        graph.replay()
        end.record()
        end.synchronize()
        torch.cuda.synchronize()
        comm.barrier()
        return start.elapsed_time(end)

    first = comm.max_([window()])[0]
    n = int(min(max_windows, max(5, math.ceil(min_total_ms / max(first, 1e-3)))))
    local = [window() for _ in range(n)]
    job = comm.max_(local)
    del graph
    return local, job


def time_steps(fns, steps, warmup, min_total_ms=50.0):
    """ms of `steps` calls on this GPU alone: the median of windows as in
    time_windows (the sweep rows)."""
    local, _ = time_windows(fns, steps, warmup, Comm(1, 0, "cpu"), min_total_ms)
    return statistics.median(local)


# ------------------------------------------------------------ CPU baseline
def cpu_reference_timing(M, K, N, seconds, threads=None):
    """The reference's CPU path, linear(SimpleRMSNorm(x)) in bf16 (oracle port),
    timed on this host's cores for about `seconds` of work."""
    import torch

    from oracle import rmsnorm_linear as orc

    threads = threads or os.cpu_count()
    torch.set_num_threads(threads)
    x, gamma, W = orc.make_inputs(M, K, N, seed=1234)
    orc.unfused_reference(x, gamma, W, None, EPS)  # warm
    n, t0 = 0, time.perf_counter()
    while True:
        orc.unfused_reference(x, gamma, W, None, EPS)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds or n >= 100000:
            break
    per_call = el / n
    return {"value": flops_of(M, K, N) / per_call / 1e12, "unit": "TFLOP/s",
            "cores": torch.get_num_threads(), "kind": "port", "us_per_call": per_call * 1e6,
            "sample": f"{n} full calls of linear(SimpleRMSNorm(x)) at {M}x{K}->{N} bf16 "
                      f"in {el:.1f} s on {torch.get_num_threads()} threads"}


def run_reference(args):
    """--impl reference: the reference's own CPU implementation of the path
    (oracle port of linear(SimpleRMSNorm(x)), bf16, all host threads).  A step
    is one full call on the workload; the K-step window is repeated until about
    two seconds have been timed and the median window is reported."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    M, K, N = SHAPES[args.config]
    import torch

    from oracle import rmsnorm_linear as orc

    torch.set_num_threads(os.cpu_count())
    x, gamma, W = orc.make_inputs(M, K, N, seed=1234)
    for _ in range(args.warmup):
        orc.unfused_reference(x, gamma, W, None, EPS)
    windows, total = [], 0.0
    while len(windows) < 5 or (total < 2.0 and len(windows) < 1000):
        t0 = time.perf_counter()
        for _ in range(args.steps):
            orc.unfused_reference(x, gamma, W, None, EPS)
        el = time.perf_counter() - t0
        windows.append(el)
        total += el
    el = statistics.median(windows)
    value = flops_of(M, K, N) * args.steps / el / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": el * 1e3 / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: x~N(0,1), gamma~1+0.1N(0,1), W~N(0,1/K) (gamma folded), "
                "seeded; no checkpoint",
        "config": make_config(args.config, args.gpus),
        "timing": {"windows": len(windows), "window_ms": spread([w * 1e3 for w in windows]),
                   "method": "perf_counter around K full calls per window, median window",
                   "path": "reference CPU torch path linear(SimpleRMSNorm(x)) (oracle port), "
                           "rank 0 only"},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": torch.get_num_threads(),
                         "kind": "port",
                         "sample": f"{len(windows)} windows of {args.steps} full calls at "
                                   f"{M}x{K}->{N}, {total:.1f} s in all"},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------- ours
def run_ours(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", device_id=device,
                                timeout=datetime.timedelta(seconds=300))
    comm = Comm(world, local_rank, device)
    global LOCAL
    LOCAL = Comm(1, local_rank, device)

    from src.load_cuda import denominator_cuda

    M, K, N = SHAPES[args.config]
    rot = Rotation(M, K, N, device, seed=1234 + 1000 * rank)
    fns = [
        (lambda i=i: denominator_cuda.fused_rmsnorm_linear(rot.xs[i], rot.wf[i], None, EPS,
                                                           rot.outs[i]))
        for i in range(rot.S)
    ]
    with ClockSampler(local_rank) as clocks:
        local, job = time_windows(fns, args.steps, args.warmup, comm, args.min_timed_ms)
    ms = statistics.median(job)
    flops = flops_of(M, K, N)
    value = world * flops * args.steps / (ms / 1e3) / 1e12
    per_launch_s = ms / 1e3 / args.steps
    rank_us = comm.gather(statistics.median(local) * 1e3 / args.steps)

    e2e = run_e2e(args, denominator_cuda, rot, comm, device, M, K, N, world)

    hbm_gbs, tflops_peak, peak_src = read_peaks()
    roof_time = max(flops / (tflops_peak * 1e12), bytes_of(M, K, N) / (hbm_gbs * 1e9))
    bound = "tensor" if flops / (tflops_peak * 1e12) >= bytes_of(M, K, N) / (hbm_gbs * 1e9) \
        else "hbm"
    if bound == "tensor":
        achieved, peak, unit = flops / per_launch_s / 1e12, tflops_peak, "TFLOP/s"
    else:
        achieved, peak, unit = bytes_of(M, K, N) / per_launch_s / 1e9, hbm_gbs, "GB/s"
    roofline = {"bound": bound, "achieved": achieved, "peak": peak, "unit": unit,
                "frac": achieved / peak, "traffic": read_profiled_traffic(
                    "fused_rmsnorm_linear" if M > 128 else "fused_rmsnorm_linear_decode",
                    args.config),
                "peak_source": f"{peak_src} (MEASURED_PEAKS.json burst figures)"
                if peak_src == "measured" else "fallback",
                "roofline_frac_of_max_time": roof_time / per_launch_s,
                "kernel": ("fused_rmsnorm_linear_pair_kernel" if M > 128
                           else "fused_rmsnorm_linear_decode_kernel"),
                "algorithmic_bytes_per_launch": bytes_of(M, K, N),
                "algorithmic_flops_per_launch": flops}

    partitioned = {}
    if not args.no_partitioned:
        partitioned["long_prefill"] = run_long_prefill(args, denominator_cuda, comm, device,
                                                       rank, world, hbm_gbs, tflops_peak)
        partitioned["int8_stack"] = run_int8_stack(args, denominator_cuda, comm, device, rank,
                                                   world, hbm_gbs, tflops_peak)

    sweep = None
    if rank == 0 and world == 1 and not args.no_sweep:
        sweep = run_sweep(denominator_cuda, device, hbm_gbs, tflops_peak)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_reference_timing(M, K, N, args.cpu_seconds)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: x~N(0,1), gamma~1+0.1N(0,1), W~N(0,1/K) (gamma folded), "
                    "seeded; no checkpoint",
            "config": make_config(args.config, world),
            "timing": {"windows": len(job), "us_per_call": ms * 1e3 / args.steps,
                       "window_ms_max_over_ranks": spread(job),
                       "us_per_call_by_rank": spread(rank_us),
                       "method": "one CUDA graph of the K calls replayed per window, CUDA "
                                 "events on the launching stream, barrier + synchronize "
                                 "around each window; median over windows of the max over "
                                 "ranks",
                       "l2": rot.describe()},
            "e2e": e2e,
            "gpu_launches": args.steps * len(job),
            "gpu_launches_detail": "fused_rmsnorm_linear_pair_kernel, K per window x windows "
                                   "of the headline timed region (one per step)",
            "roofline": roofline,
            "cpu_baseline": cpu,
            "clocks": clocks.summary(),
        }
        line.update(partitioned)
        if sweep is not None:
            line["sweep"] = sweep
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()


def run_e2e(args, denominator_cuda, rot, comm, device, M, K, N, world):
    """The headline metric end to end through the public API with pinned host
    buffers: every step copies its x in from pinned host memory, runs the op
    and copies its whole output back.  Steps are pipelined the way a server
    overlaps requests: copy-in, compute and copy-out on three streams, two
    buffer sets, so step i's device-to-host read overlaps step i+1's copy-in
    and kernel.  Windows of K steps, median of the max over ranks."""
    import torch

    flops = flops_of(M, K, N)
    x_host = rot.xs[0].cpu().pin_memory()
    out_host = [torch.empty(M, N, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    xd = [torch.empty_like(rot.xs[0]) for _ in range(2)]
    od = [torch.empty(M, N, dtype=torch.bfloat16, device=device) for _ in range(2)]
    s_in, s_cmp, s_out = (torch.cuda.Stream(device) for _ in range(3))
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_cmp = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]

    def e2e_step(i):
        j = i % 2
        with torch.cuda.stream(s_in):
            s_in.wait_event(ev_cmp[j])  # the kernel that read xd[j] two steps ago
            xd[j].copy_(x_host, non_blocking=True)
            ev_in[j].record(s_in)
        with torch.cuda.stream(s_cmp):
            s_cmp.wait_event(ev_in[j])
            s_cmp.wait_event(ev_out[j])  # the read-back of od[j] two steps ago
            denominator_cuda.fused_rmsnorm_linear(xd[j], rot.wf[0], None, EPS, od[j])
            ev_cmp[j].record(s_cmp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_cmp[j])
            out_host[j].copy_(od[j], non_blocking=True)
            ev_out[j].record(s_out)

    cur = torch.cuda.current_stream(device)
    for i in range(max(4, args.warmup)):
        e2e_step(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def window():
        comm.barrier()
        torch.cuda.synchronize()
        e0.record(cur)
        for st in (s_in, s_cmp, s_out):
            st.wait_event(e0)
        for i in range(args.steps):
            e2e_step(i)
        for st in (s_in, s_cmp, s_out):
            cur.wait_stream(st)
        e1.record(cur)
        e1.synchronize()
        comm.barrier()
        return e0.elapsed_time(e1)

    first = comm.max_([window()])[0]
    n = int(min(500, max(5, math.ceil(args.min_timed_ms / max(first, 1e-3)))))
    local = [window() for _ in range(n)]
    job = comm.max_(local)
    ms = statistics.median(job)
    step_us_by_rank = comm.gather(statistics.median(local) * 1e3 / args.steps)
    d2h = M * N * 2
    return {"value": world * flops * args.steps / (ms / 1e3) / 1e12, "unit": "TFLOP/s",
            "h2d_bytes_per_step": M * K * 2, "d2h_bytes_per_step": d2h,
            "steps": args.steps, "windows": n,
            "us_per_step_by_rank": spread(step_us_by_rank),
            "d2h_gbs_per_rank": spread([d2h / us / 1e3 for us in step_us_by_rank]),
            "path": "denominator_cuda.fused_rmsnorm_linear, pinned host x -> HBM, out -> "
                    "pinned host, W resident; copy-in / kernel / copy-out on three streams, "
                    "two buffer sets (step i's read-back overlaps step i+1)"}


def run_long_prefill(args, denominator_cuda, comm, device, rank, world, hbm_gbs, tflops_peak):
    """q_b and kv_b at 4096 tokens in total, token-partitioned: rank r takes its
    contiguous share of the rows (4096 / N) against its own replica of W (the
    same W on every rank), no collective.  Reports the job time (median window
    of the max over ranks) against the per-GPU roofline of the busiest rank,
    and, on rank 0, the whole 4096 rows on one GPU for the strong-scaling
    ratio."""
    import torch

    from src.multigpu import shard_bounds

    res = {}
    steps = 20
    for name, (M_tot, K, N) in LONG_PREFILL.items():
        s, e = shard_bounds(M_tot, world, rank)
        m = e - s
        rot = Rotation(m, K, N, device, seed=4000 + 1000 * rank, w_seed=9000)
        fns = [(lambda i=i: denominator_cuda.fused_rmsnorm_linear(rot.xs[i], rot.wf[i], None,
                                                                  EPS, rot.outs[i]))
               for i in range(rot.S)]
        local, job = time_windows(fns, steps, 3, comm, 100.0)
        job_us = statistics.median(job) * 1e3 / steps
        rank_us = comm.gather(statistics.median(local) * 1e3 / steps)
        m_max = max(shard_bounds(M_tot, world, r)[1] - shard_bounds(M_tot, world, r)[0]
                    for r in range(world))
        roof = roofline_us(flops_of(m_max, K, N), bytes_of(m_max, K, N), hbm_gbs, tflops_peak)
        del rot, fns
        torch.cuda.empty_cache()
        one_gpu_us = None
        if world > 1:
            comm.barrier()
            if rank == 0:  # the same total on one GPU, for the strong-scaling ratio
                r1 = Rotation(M_tot, K, N, device, seed=4000, w_seed=9000)
                f1 = [(lambda i=i: denominator_cuda.fused_rmsnorm_linear(
                    r1.xs[i], r1.wf[i], None, EPS, r1.outs[i])) for i in range(r1.S)]
                l1, _ = time_windows(f1, steps, 3, LOCAL, 100.0)
                one_gpu_us = statistics.median(l1) * 1e3 / steps
                del r1, f1
                torch.cuda.empty_cache()
            comm.barrier()
        res[name] = {
            "tokens_total": M_tot, "tokens_per_rank": m_max, "hidden": K, "out": N,
            "job_us": round(job_us, 3), "us_by_rank": spread(rank_us),
            "tflops_job": round(flops_of(M_tot, K, N) / job_us / 1e6, 1),
            "roofline_us_per_gpu": round(roof, 3), "frac_of_roofline": round(roof / job_us, 3),
            "one_gpu_us": round(one_gpu_us, 3) if one_gpu_us else None,
            "strong_scaling_efficiency": (round(one_gpu_us / (world * job_us), 3)
                                          if one_gpu_us else None),
        }
    return res


def run_int8_stack(args, denominator_cuda, comm, device, rank, world, hbm_gbs, tflops_peak):
    """61 Kimi layers of int8 q_b (1536 -> 12288) + int8 kv_b (512 -> 16384) at
    2048 tokens in total, token-partitioned: rank r runs its share of the rows
    through all 122 projections, a layer's q_b and kv_b in one grouped launch
    (61 launches; weights quantized per output channel, replicated
    and identical on every rank; every layer has its own x and output buffer,
    several GB in all, so nothing stays in L2 from one stack to the next).  One
    step = one whole stack, replayed from a CUDA graph."""
    import torch

    from src.multigpu import shard_bounds

    s, e = shard_bounds(STACK_TOKENS, world, rank)
    m = e - s
    layers, xs, outs = [], [], []
    for li in range(STACK_LAYERS):
        for si, (_, K, N) in enumerate(STACK_SHAPES):
            _, gamma, W = gpu_inputs(1, K, N, 20000 + 10 * li + si, device)
            q, sc = denominator_cuda.quantize_int8_per_channel(W * gamma)
            del W
            layers.append(((q, sc), None))
            g = torch.Generator(device=device).manual_seed(30000 + 1000 * rank + 10 * li + si)
            xs.append(torch.randn(m, K, generator=g, device=device).to(torch.bfloat16))
            outs.append(torch.empty(m, N, dtype=torch.bfloat16, device=device))
    torch.cuda.synchronize()

    def stack():
        # The launches fused_stack_token_parallel makes, each writing into this
        # rank's own preallocated outputs: a layer's q_b and kv_b in one
        # grouped launch (independent inputs).
        for li in range(0, len(layers), 2):
            (qa, sa), ba = layers[li]
            (qb, sb), bb = layers[li + 1]
            denominator_cuda.fused_rmsnorm_linear_w8_grouped(
                xs[li], qa, sa, ba, xs[li + 1], qb, sb, bb, EPS, outs[li], outs[li + 1])

    local, job = time_windows([stack], 1, 2, comm, 100.0, max_windows=200)
    job_us = statistics.median(job) * 1e3
    rank_us = comm.gather(statistics.median(local) * 1e3)
    m_max = max(shard_bounds(STACK_TOKENS, world, r)[1] - shard_bounds(STACK_TOKENS, world, r)[0]
                for r in range(world))
    roof = STACK_LAYERS * sum(roofline_us(flops_of(m_max, K, N), bytes_of_w8(m_max, K, N),
                                          hbm_gbs, tflops_peak) for _, K, N in STACK_SHAPES)
    fl = STACK_LAYERS * sum(flops_of(STACK_TOKENS, K, N) for _, K, N in STACK_SHAPES)
    del layers, xs, outs
    torch.cuda.empty_cache()
    return {"layers": STACK_LAYERS, "tokens_total": STACK_TOKENS, "tokens_per_rank": m_max,
            "launches_per_stack": STACK_LAYERS,
            "launch": "one grouped int8 launch per layer (q_b and kv_b)",
            "job_us_per_stack": round(job_us, 3), "us_by_rank": spread(rank_us),
            "us_per_layer_pair": round(job_us / STACK_LAYERS, 3),
            "tflops_job": round(fl / job_us / 1e6, 1),
            "roofline_us_per_stack": round(roof, 3), "frac_of_roofline": round(roof / job_us, 3)}


def run_sweep(denominator_cuda, device, hbm_gbs, tflops_peak, steps=400):
    """µs/call of every BASELINE shape: ours, the unfused cuBLAS path, the
    reference's fused path (cuBLAS F.linear + the in-place normalize epilogue)
    and the cuBLAS GEMM alone;
    cold (rotating sets larger than L2; the roofline fraction uses this) and
    hot (one set reused, L2-warm where it fits)."""
    import torch

    res = {}
    for name, (M, K, N) in SHAPES.items():
        rot = Rotation(M, K, N, device, seed=99)
        ours = [(lambda i=i: denominator_cuda.fused_rmsnorm_linear(rot.xs[i], rot.wf[i], None,
                                                                   EPS, rot.outs[i]))
                for i in range(rot.S)]
        base = [(lambda i=i: unfused_torch(rot.xs[i], rot.gammas[i], rot.ws[i], EPS))
                for i in range(rot.S)]
        # The reference's fused path, F.linear(x, W_new) then the in-place
        # normalize epilogue (src/fused_forward.py:182-191 there), with this
        # library's normalize kernel; and the library GEMM alone.
        zb = torch.zeros(N, dtype=torch.bfloat16, device=device)

        def ref_path(i):
            raw = torch.nn.functional.linear(rot.xs[i], rot.wf[i])
            denominator_cuda.rmsnorm_normalize_512(rot.xs[i], raw, zb, K, EPS)

        refp = [(lambda i=i: ref_path(i)) for i in range(rot.S)]
        gemm = [(lambda i=i: torch.nn.functional.linear(rot.xs[i], rot.wf[i]))
                for i in range(rot.S)]
        n = max(rot.S, min(steps, 4 * rot.S))
        t_ours = time_steps(ours, n, rot.S) * 1e3 / n
        t_base = time_steps(base, n, rot.S) * 1e3 / n
        t_refp = time_steps(refp, n, rot.S) * 1e3 / n
        t_gemm = time_steps(gemm, n, rot.S) * 1e3 / n
        # Hot: the same set every call, so whatever of it fits stays in L2.
        t_hot = time_steps(ours[:1], n, rot.S) * 1e3 / n
        fl, by = flops_of(M, K, N), bytes_of(M, K, N)
        roof_us = max(fl / (tflops_peak * 1e12), by / (hbm_gbs * 1e9)) * 1e6
        res[name] = {"us_per_call": round(t_ours, 3), "tflops": round(fl / t_ours / 1e6, 1),
                     "gbs": round(by / t_ours / 1e3, 1),
                     "roofline_us": round(roof_us, 3), "frac_of_roofline": round(roof_us / t_ours, 3),
                     "us_per_call_hot_l2": round(t_hot, 3),
                     "unfused_cublas_us": round(t_base, 3),
                     "speedup_vs_unfused": round(t_base / t_ours, 3),
                     "reference_fused_path_us": round(t_refp, 3),
                     "speedup_vs_reference_fused_path": round(t_refp / t_ours, 3),
                     "cublas_gemm_only_us": round(t_gemm, 3)}
        del rot
        torch.cuda.empty_cache()
    res["int8_q_b"] = sweep_int8(denominator_cuda, device, hbm_gbs, tflops_peak, steps)
    for name, M in (("swiglu_llama_prefill", 512), ("swiglu_llama_decode_m8", 8)):
        res[name] = sweep_swiglu(denominator_cuda, device, hbm_gbs, tflops_peak, M, steps)
    res["gqa_decode_llama"] = sweep_gqa(denominator_cuda, device, hbm_gbs, steps)
    return res


def sweep_swiglu(denominator_cuda, device, hbm_gbs, tflops_peak, M, steps):
    """Llama-3-8B MLP gate/up (K=4096, I=14336): one fused launch vs the
    reference's FusedRMSNormSwiGLU path (F.linear over W_combined, then its
    rmsnorm_swiglu epilogue) on the same GPU."""
    import torch
    import torch.nn.functional as F

    K, inter = 4096, 14336
    sets = []
    for s in range(2):  # 2 x 235 MB of weights > L2
        x, gamma, W = gpu_inputs(M, K, 2 * inter, 700 + s, device)
        Wc = (W * gamma).contiguous()
        b = torch.zeros(2 * inter, dtype=torch.bfloat16, device=device)
        sets.append((x, Wc, b, torch.empty(M, inter, dtype=torch.bfloat16, device=device)))
    ours = [(lambda t=t: denominator_cuda.fused_rmsnorm_swiglu(t[0], t[1], None, EPS, t[3]))
            for t in sets]

    def ref_path(t):
        x, Wc, b, out = t
        denominator_cuda.rmsnorm_swiglu(x, F.linear(x, Wc), out, b, K, inter, EPS)

    base = [(lambda t=t: ref_path(t)) for t in sets]
    n = 40
    t_ours = time_steps(ours, n, 2) * 1e3 / n
    t_base = time_steps(base, n, 2) * 1e3 / n
    fl = 2.0 * M * K * 2 * inter
    by = 2.0 * (M * K + 2 * inter * K + M * inter)
    roof_us = max(fl / (tflops_peak * 1e12), by / (hbm_gbs * 1e9)) * 1e6
    return {"us_per_call": round(t_ours, 3), "roofline_us": round(roof_us, 3),
            "frac_of_roofline": round(roof_us / t_ours, 3),
            "reference_linear_then_swiglu_us": round(t_base, 3),
            "speedup_vs_reference_path": round(t_base / t_ours, 3)}


def sweep_gqa(denominator_cuda, device, hbm_gbs, steps):
    """Decode-step GQA attention, Llama-3-8B heads (32 q / 8 kv, d 128) at
    batch 4 over a 4096-token cache: ours vs SDPA over repeated KV heads."""
    import torch
    import torch.nn.functional as F

    B, Hq, Hkv, D, T = 4, 32, 8, 128, 4096
    g = torch.Generator(device=device).manual_seed(5)
    sets = []
    for s in range(4):  # 4 x 67 MB of K/V > L2
        q = torch.randn(B, Hq, D, generator=g, device=device).to(torch.bfloat16)
        k = torch.randn(B, T, Hkv, D, generator=g, device=device).to(torch.bfloat16)
        v = torch.randn(B, T, Hkv, D, generator=g, device=device).to(torch.bfloat16)
        sets.append((q, k, v, torch.empty_like(q)))
    scale = 1.0 / math.sqrt(D)
    ours = [(lambda t=t: denominator_cuda.gqa_decode_v3(t[0], t[1], t[2], t[3], Hq // Hkv, scale))
            for t in sets]

    def sdpa(t):
        q, k, v, _ = t
        kk = k.repeat_interleave(Hq // Hkv, dim=2).permute(0, 2, 1, 3)
        vv = v.repeat_interleave(Hq // Hkv, dim=2).permute(0, 2, 1, 3)
        return F.scaled_dot_product_attention(q.unsqueeze(2), kk, vv, scale=scale)

    base = [(lambda t=t: sdpa(t)) for t in sets]
    n = 40
    t_ours = time_steps(ours, n, 4) * 1e3 / n
    t_base = time_steps(base, n, 4) * 1e3 / n
    by = 2.0 * (2 * B * T * Hkv * D + 2 * B * Hq * D)
    roof_us = by / (hbm_gbs * 1e9) * 1e6
    return {"us_per_call": round(t_ours, 3), "roofline_us": round(roof_us, 3),
            "frac_of_roofline": round(roof_us / t_ours, 3), "sdpa_repeat_kv_us": round(t_base, 3),
            "speedup_vs_sdpa": round(t_base / t_ours, 3)}


def sweep_int8(denominator_cuda, device, hbm_gbs, tflops_peak, steps):
    """int8-weight q_b at 2048 tokens: ours vs the reference's quantization-
    aware GPU path (dequantize W to bf16, then F.linear(x * bf16(inv_rms), W))."""
    import torch
    import torch.nn.functional as F

    M, K, N = 2048, 1536, 12288
    sets = []
    for s in range(4):
        x, gamma, W = gpu_inputs(M, K, N, 500 + s, device)
        q, sc = denominator_cuda.quantize_int8_per_channel(W * gamma)
        sets.append((x, q, sc, torch.empty(M, N, dtype=torch.bfloat16, device=device)))
    ours = [(lambda t=t: denominator_cuda.fused_rmsnorm_linear_w8(t[0], t[1], t[2], None, EPS, t[3]))
            for t in sets]

    def ref_path(t):
        x, q, sc, _ = t
        w = (q.float() * sc.float().unsqueeze(1)).to(torch.bfloat16)
        variance = x.float().pow(2).mean(dim=-1, keepdim=True)
        return F.linear(x * torch.rsqrt(variance + EPS).to(torch.bfloat16), w)

    base = [(lambda t=t: ref_path(t)) for t in sets]
    n = 16
    t_ours = time_steps(ours, n, 4) * 1e3 / n
    t_base = time_steps(base, n, 4) * 1e3 / n
    fl = flops_of(M, K, N)
    by = M * K * 2 + N * K + N * 4 + M * N * 2
    roof_us = max(fl / (tflops_peak * 1e12), by / (hbm_gbs * 1e9)) * 1e6
    return {"us_per_call": round(t_ours, 3), "tflops": round(fl / t_ours / 1e6, 1),
            "roofline_us": round(roof_us, 3), "frac_of_roofline": round(roof_us / t_ours, 3),
            "reference_dequant_linear_us": round(t_base, 3),
            "speedup_vs_reference_path": round(t_base / t_ours, 3)}


def run_profile(args):
    """--profile CASE: CASE's fused kernel launched --warmup + --steps times
    eagerly on cuda:0 with no timing (for ncu: -k picks the kernel, -s skips
    the warm-up launches).  Linear shapes rotate over sets larger than L2."""
    import torch

    from src.load_cuda import denominator_cuda

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    n = args.warmup + args.steps
    case = args.profile
    if case in SHAPES:
        M, K, N = SHAPES[case]
        rot = Rotation(M, K, N, device, seed=99)
        for i in range(n):
            j = i % rot.S
            denominator_cuda.fused_rmsnorm_linear(rot.xs[j], rot.wf[j], None, EPS, rot.outs[j])
    elif case == "int8_layer_256":
        # one 8-GPU shard of the int8 stack's layer: q_b and kv_b at 256 rows,
        # one grouped launch
        sets = []
        for s in range(4):
            row = []
            for K, N in ((1536, 12288), (512, 16384)):
                x, gamma, W = gpu_inputs(256, K, N, 600 + 2 * s + len(row), device)
                q, sc = denominator_cuda.quantize_int8_per_channel(W * gamma)
                row.append((x, q, sc, torch.empty(256, N, dtype=torch.bfloat16, device=device)))
            sets.append(row)
        for i in range(n):
            (xa, qa, sa, oa), (xb, qb, sb, ob) = sets[i % 4]
            denominator_cuda.fused_rmsnorm_linear_w8_grouped(xa, qa, sa, None, xb, qb, sb, None,
                                                             EPS, oa, ob)
    elif case.startswith("int8_"):
        M, K, N = {"int8_q_b": (2048, 1536, 12288), "int8_q_b_256": (256, 1536, 12288),
                   "int8_kv_b_256": (256, 512, 16384)}[case]
        sets = []
        for s in range(4):
            x, gamma, W = gpu_inputs(M, K, N, 500 + s, device)
            q, sc = denominator_cuda.quantize_int8_per_channel(W * gamma)
            sets.append((x, q, sc, torch.empty(M, N, dtype=torch.bfloat16, device=device)))
        for i in range(n):
            x, q, sc, o = sets[i % 4]
            denominator_cuda.fused_rmsnorm_linear_w8(x, q, sc, None, EPS, o)
    elif case.startswith("swiglu_"):
        M = 512 if case == "swiglu_prefill" else 8
        K, inter = 4096, 14336
        sets = []
        for s in range(2):
            x, gamma, W = gpu_inputs(M, K, 2 * inter, 700 + s, device)
            sets.append((x, (W * gamma).contiguous(),
                         torch.empty(M, inter, dtype=torch.bfloat16, device=device)))
        for i in range(n):
            x, Wc, o = sets[i % 2]
            denominator_cuda.fused_rmsnorm_swiglu(x, Wc, None, EPS, o)
    else:  # gqa_decode_llama
        hbm_gbs, _, _ = read_peaks()
        print(json.dumps({"gqa_decode_llama": sweep_gqa(denominator_cuda, device, hbm_gbs, n)}))
    torch.cuda.synchronize()
    print(json.dumps({"profile": case, "launches": n}), flush=True)


def main():
    args = parse_args()
    if args.gqa_only:
        args.profile = "gqa_decode_llama"
    if args.profile:
        run_profile(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
