#!/usr/bin/env python
"""Benchmark of the fused RMSNorm -> Linear hot path (Kimi K2.6 kv_b shape).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step is one fused RMSNorm -> Linear call over one 512-token batch of the
kimi_kv_b workload (x [512, 512] bf16, W_fused [16384, 512], out [512, 16384]).
Steps rotate over enough (x, W, out) buffer sets that the working set is
about twice the 126 MB L2, so every call streams W and out from/to HBM.  The
K timed steps are replayed from CUDA graphs (one node per call), bracketed by a
barrier and torch.cuda.synchronize() on both sides, timed with CUDA events on
the launching stream; the max over ranks is reported.  With N > 1 (torchrun,
one rank per GPU) each rank processes its own 512-token shard with its own
weight replica and there is no collective on the data path (weak scaling).

One JSON line is printed by rank 0; see DESIGN.md for every key.
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


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(SHAPES), default=HEADLINE)
    ap.add_argument("--no-sweep", action="store_true", help="skip the per-config sweep")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--gqa-only", action="store_true",
                    help="time only the GQA decode-attention workload (one JSON line; for profiling)")
    return ap.parse_args()


def flops_of(M, K, N):
    return 2.0 * M * K * N


def bytes_of(M, K, N, elem=2):
    return float(elem) * (M * K + N * K + M * N)


def read_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, 1590.0, "fallback"


def read_profiled_traffic(kernel: str, workload: str):
    """Per-launch DRAM bytes recorded from an ncu capture in profiles/."""
    path = os.path.join(REPO, "profiles", f"{kernel}__{workload}.md")
    try:
        text = open(path).read()
    except OSError:
        return None
    m = re.search(r"traffic_bytes_per_launch\s*[:=]\s*([0-9.eE+]+)", text)
    return float(m.group(1)) if m else None


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

    def __init__(self, M, K, N, device, seed=1234, min_sets=2):
        import torch

        set_bytes = bytes_of(M, K, N)
        self.S = max(min_sets, int(math.ceil(2 * L2_BYTES / set_bytes)))
        self.xs, self.gammas, self.ws, self.wf, self.outs = [], [], [], [], []
        for s in range(self.S):
            x, gamma, W = gpu_inputs(M, K, N, seed + s, device)
            self.xs.append(x)
            self.gammas.append(gamma)
            self.ws.append(W)
            self.wf.append(W * gamma)
            self.outs.append(torch.empty(M, N, dtype=torch.bfloat16, device=device))
        self.set_bytes = set_bytes

    def describe(self):
        tot = self.S * self.set_bytes
        return f"rotating {self.S} (x, W, out) sets, {tot / 1e6:.0f} MB > 126 MB L2"


def time_steps(fns, steps, warmup, barrier=None):
    """Run `steps` calls fns[i % S], replayed from CUDA graphs; returns the
    elapsed ms of exactly `steps` calls (events on the launching stream)."""
    import torch

    S = len(fns)
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        for f in fns:  # eager warm call: attributes, tensor-map entry point
            f()
    torch.cuda.current_stream().wait_stream(stream)
    torch.cuda.synchronize()
    full = torch.cuda.CUDAGraph()
    with torch.cuda.graph(full):
        for f in fns:
            f()
    rem = steps % S
    part = None
    if rem:
        part = torch.cuda.CUDAGraph()
        with torch.cuda.graph(part):
            for f in fns[:rem]:
                f()
    for _ in range(max(1, math.ceil(warmup / S))):
        full.replay()
    torch.cuda.synchronize()
    if barrier:
        barrier()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps // S):
        full.replay()
    if part is not None:
        part.replay()
    end.record()
    end.synchronize()
    torch.cuda.synchronize()
    if barrier:
        barrier()
    ms = start.elapsed_time(end)
    del full, part
    return ms


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
    (oracle port of linear(SimpleRMSNorm(x)), bf16, all host threads)."""
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
    t0 = time.perf_counter()
    for _ in range(args.steps):
        orc.unfused_reference(x, gamma, W, None, EPS)
    el = time.perf_counter() - t0
    value = flops_of(M, K, N) * args.steps / el / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": el * 1e3 / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: x~N(0,1), gamma~1+0.1N(0,1), W~N(0,1/K), seed 1234",
        "config": {"workload": args.config, "tokens": M, "hidden": K, "out": N,
                   "path": "reference CPU torch path linear(SimpleRMSNorm(x)) (oracle port)"},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": torch.get_num_threads(),
                         "kind": "port",
                         "sample": f"{args.steps} full calls at {M}x{K}->{N}"},
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
        barrier = lambda: dist.barrier(device_ids=[local_rank])  # noqa: E731
    else:
        barrier = None

    from src.load_cuda import denominator_cuda

    M, K, N = SHAPES[args.config]
    rot = Rotation(M, K, N, device, seed=1234 + 1000 * rank)
    fns = [
        (lambda i=i: denominator_cuda.fused_rmsnorm_linear(rot.xs[i], rot.wf[i], None, EPS,
                                                           rot.outs[i]))
        for i in range(rot.S)
    ]
    with ClockSampler(local_rank) as clocks:
        ms = time_steps(fns, args.steps, args.warmup, barrier)
    t = torch.tensor([ms], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    flops = flops_of(M, K, N)
    value = world * flops * args.steps / (ms / 1e3) / 1e12
    per_launch_s = ms / 1e3 / args.steps

    # ---- e2e through the public API with pinned host buffers.  Every step
    # copies its x in from pinned host memory, runs the op and copies its whole
    # output back; steps are pipelined the way a server overlaps requests:
    # copy-in, compute and copy-out on three streams, two buffer sets, so step
    # i's device-to-host read overlaps step i+1's copy-in and kernel.
    e2e_steps = max(1, min(args.steps, 200))
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
    for i in range(4):
        e2e_step(i)
    torch.cuda.synchronize()
    if barrier:
        barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(cur)
    for st in (s_in, s_cmp, s_out):
        st.wait_event(e0)
    for i in range(e2e_steps):
        e2e_step(i)
    for st in (s_in, s_cmp, s_out):
        cur.wait_stream(st)
    e1.record(cur)
    e1.synchronize()
    te = torch.tensor([e0.elapsed_time(e1)], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_value = world * flops * e2e_steps / (float(te.item()) / 1e3) / 1e12

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
            "config": {"workload": args.config, "tokens_per_gpu": M, "hidden": K, "out": N,
                       "parallelism": f"token-partitioned x{world}, replicated W, "
                                      "no collective" if world > 1 else "single GPU",
                       "l2": rot.describe(), "timing": "CUDA graph replay of K calls, "
                                                       "CUDA events on the launching stream",
                       "us_per_call": ms * 1e3 / args.steps},
            "e2e": {"value": e2e_value, "unit": "TFLOP/s",
                    "h2d_bytes_per_step": M * K * 2, "d2h_bytes_per_step": M * N * 2,
                    "steps": e2e_steps,
                    "path": "denominator_cuda.fused_rmsnorm_linear, pinned host x -> HBM, "
                            "out -> pinned host, W resident; copy-in / kernel / copy-out "
                            "on three streams, two buffer sets (step i's read-back "
                            "overlaps step i+1)"},
            "gpu_launches": args.steps,
            "roofline": roofline,
            "cpu_baseline": cpu,
            "clocks": clocks.summary(),
        }
        if sweep is not None:
            line["sweep"] = sweep
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()


def run_sweep(denominator_cuda, device, hbm_gbs, tflops_peak, steps=400):
    """µs/call of every BASELINE shape (ours vs the unfused cuBLAS path):
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
        n = max(rot.S, min(steps, 4 * rot.S))
        t_ours = time_steps(ours, n, rot.S) * 1e3 / n
        t_base = time_steps(base, n, rot.S) * 1e3 / n
        # Hot: the same set every call, so whatever of it fits stays in L2.
        t_hot = time_steps(ours[:1], n, rot.S) * 1e3 / n
        fl, by = flops_of(M, K, N), bytes_of(M, K, N)
        roof_us = max(fl / (tflops_peak * 1e12), by / (hbm_gbs * 1e9)) * 1e6
        res[name] = {"us_per_call": round(t_ours, 3), "tflops": round(fl / t_ours / 1e6, 1),
                     "gbs": round(by / t_ours / 1e3, 1),
                     "roofline_us": round(roof_us, 3), "frac_of_roofline": round(roof_us / t_ours, 3),
                     "us_per_call_hot_l2": round(t_hot, 3),
                     "unfused_cublas_us": round(t_base, 3),
                     "speedup_vs_unfused": round(t_base / t_ours, 3)}
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


def main():
    args = parse_args()
    if args.gqa_only:
        import torch
        from src.load_cuda import denominator_cuda
        hbm_gbs, _, _ = read_peaks()
        print(json.dumps({"gqa_decode_llama": sweep_gqa(
            denominator_cuda, torch.device("cuda"), hbm_gbs, 40)}))
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
