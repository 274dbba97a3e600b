"""Kimi K2.6 fused RMSNorm -> Linear benchmark (same CLI and key=value output
as the reference's src/benchmark_kimi26.py:44-111).

    python -m src.benchmark_kimi26 --config kimi_kv_b --variant V3

Builds SimpleRMSNorm (gamma = ones, as the reference) and an nn.Linear with
torch's default init at seed 1234, folds gamma into the weight, and times the
unfused baseline linear(norm(x)) against the fused module.  Timing is the
reference's wall-clock method (perf_counter around `iters` calls with a device
synchronize at each end); ``--cuda-events`` times on the stream instead.
"""

from __future__ import annotations

import argparse
import time

import torch
import torch.nn as nn

from src.fused_forward import FusedRMSNormLinearV1, FusedRMSNormLinearV3
from src.weight_transform import compute_fused_weights_rmsnorm


class SimpleRMSNorm(nn.Module):
    """x * rsqrt(mean(x^2) + eps) (cast to x's dtype) * weight, the norm the
    reference benchmarks against (reference src/benchmark_kimi26.py:23-31)."""

    def __init__(self, hidden_size: int, eps: float = 1e-5):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(hidden_size))
        self.variance_epsilon = eps

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        variance = x.float().pow(2).mean(dim=-1, keepdim=True)
        return x * torch.rsqrt(variance + self.variance_epsilon).to(x.dtype) * self.weight.to(x.dtype)


CONFIGS = {
    "kimi_q_b": {"tokens": 512, "hidden": 1536, "out": 12288},
    "kimi_kv_b": {"tokens": 512, "hidden": 512, "out": 16384},
    "kimi_q_b_long": {"tokens": 4096, "hidden": 1536, "out": 12288},
    "kimi_kv_b_long": {"tokens": 4096, "hidden": 512, "out": 16384},
}


def parse_args(argv=None) -> argparse.Namespace:
    p = argparse.ArgumentParser(description="Benchmark Kimi K2.6 fused RMSNorm+Linear on B200.")
    p.add_argument("--config", choices=CONFIGS.keys(), default="kimi_q_b")
    p.add_argument("--tokens", type=int)
    p.add_argument("--hidden", type=int)
    p.add_argument("--out", type=int)
    p.add_argument("--variant", choices=["V1", "V3"], default="V3")
    p.add_argument("--dtype", choices=["bfloat16", "float16", "float32"], default="bfloat16")
    p.add_argument("--warmup", type=int, default=30)
    p.add_argument("--iters", type=int, default=300)
    p.add_argument("--cuda-events", action="store_true")
    return p.parse_args(argv)


def bench(fn, x, warmup: int, iters: int, cuda_events: bool = False) -> float:
    with torch.no_grad():
        for _ in range(warmup):
            fn(x)
        torch.cuda.synchronize()
        if cuda_events:
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for _ in range(iters):
                fn(x)
            b.record()
            b.synchronize()
            return a.elapsed_time(b) / iters
        start = time.perf_counter()
        for _ in range(iters):
            fn(x)
        torch.cuda.synchronize()
    return (time.perf_counter() - start) * 1000.0 / iters


def main(argv=None) -> None:
    if not torch.cuda.is_available():
        raise SystemExit("CUDA is required for this benchmark.")
    args = parse_args(argv)
    cfg = CONFIGS[args.config]
    tokens = args.tokens or cfg["tokens"]
    hidden = args.hidden or cfg["hidden"]
    out = args.out or cfg["out"]
    dtype = getattr(torch, args.dtype)
    device = torch.device("cuda")

    torch.manual_seed(1234)
    norm = SimpleRMSNorm(hidden, eps=1e-5).to(device=device, dtype=dtype)
    linear = nn.Linear(hidden, out, bias=False).to(device=device, dtype=dtype)
    x = torch.randn(tokens, hidden, device=device, dtype=dtype)
    W_new, b_new, h, eps = compute_fused_weights_rmsnorm(norm, linear)
    cls = FusedRMSNormLinearV3 if args.variant == "V3" else FusedRMSNormLinearV1
    fused = cls(W_new.to(device), b_new.to(device), h, eps)
    baseline = lambda t: linear(norm(t))  # noqa: E731

    with torch.no_grad():
        diff = (baseline(x).float() - fused(x).float()).abs()
    baseline_ms = bench(baseline, x, args.warmup, args.iters, args.cuda_events)
    fused_ms = bench(fused, x, args.warmup, args.iters, args.cuda_events)
    flops = 2.0 * tokens * hidden * out
    print(f"config={args.config} variant={args.variant}")
    print(f"gpu={torch.cuda.get_device_name(0)} dtype={dtype}")
    print(f"shape=({tokens}, {hidden}) -> {out}")
    print(f"max_abs_diff={float(diff.max()):.6e}")
    print(f"mean_abs_diff={float(diff.mean()):.6e}")
    print(f"baseline_ms={baseline_ms:.4f}")
    print(f"fused_ms={fused_ms:.4f}")
    print(f"speedup={baseline_ms / fused_ms:.3f}x")
    print(f"fused_tflops={flops / (fused_ms * 1e-3) / 1e12:.1f}")


if __name__ == "__main__":
    main()
