"""Kimi K2.6 fused RMSNorm -> Linear benchmark with the reference's command
line and key=value output lines (reference src/benchmark_kimi26.py:44-111):

    python -m src.benchmark_kimi26 --config kimi_kv_b --variant V3

A thin driver over this repository's bench.py: the inputs are its seeded
synthetic tensors (x ~ N(0,1), gamma ~ 1 + 0.1 N(0,1), W ~ N(0, 1/K)), the
baseline is its unfused linear(SimpleRMSNorm(x)) on the GPU, and both paths
are timed the way bench.py times its sweep rows (CUDA-graph replay of the
calls, CUDA events on the launching stream, median of repeated windows).  The
fused path is the module a model patched by patch_kimi calls.
"""

from __future__ import annotations

import argparse
import os
import sys

import torch
import torch.nn as nn

from src.fused_forward import FusedRMSNormLinearV1, FusedRMSNormLinearV3

_REPO = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def bench_module():
    """The repository's bench.py (inputs, baseline and timing)."""
    if _REPO not in sys.path:
        sys.path.insert(0, _REPO)
    import bench

    return bench


class SimpleRMSNorm(nn.Module):
    """The norm the reference benchmarks against (its src/benchmark_kimi26.py:23-31):
    x * rsqrt(mean(x^2) + eps) cast to x's dtype, times the weight."""

    def __init__(self, hidden_size: int, eps: float = 1e-5):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(hidden_size))
        self.variance_epsilon = eps

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        r = torch.rsqrt(x.float().pow(2).mean(dim=-1, keepdim=True) + self.variance_epsilon)
        return x * r.to(x.dtype) * self.weight.to(x.dtype)


# The reference's four Kimi shapes (tokens, hidden, out).
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
    return p.parse_args(argv)


def time_ms(fn, warmup: int, iters: int) -> float:
    """Milliseconds per call of fn() (bench.py's single-GPU window timing)."""
    with torch.no_grad():
        return bench_module().time_steps([fn], iters, warmup) / iters


def shape_of(args) -> tuple[int, int, int]:
    cfg = CONFIGS[args.config]
    return (args.tokens or cfg["tokens"], args.hidden or cfg["hidden"], args.out or cfg["out"])


def main(argv=None) -> None:
    if not torch.cuda.is_available():
        raise SystemExit("CUDA is required for this benchmark.")
    args = parse_args(argv)
    if args.dtype == "float32":
        raise SystemExit("the fused kernels take bfloat16 or float16 activations (no fp32 path)")
    dtype = getattr(torch, args.dtype)
    tokens, hidden, out = shape_of(args)
    b = bench_module()
    x, gamma, W = (t.to(dtype) for t in b.gpu_inputs(tokens, hidden, out, 1234, "cuda"))
    cls = FusedRMSNormLinearV3 if args.variant == "V3" else FusedRMSNormLinearV1
    fused = cls(W * gamma, torch.zeros(out, dtype=dtype, device="cuda"), hidden, b.EPS)
    with torch.no_grad():
        ref = b.unfused_torch(x, gamma, W, b.EPS).float()
        diff = (ref - fused(x).float()).abs()
    baseline_ms = time_ms(lambda: b.unfused_torch(x, gamma, W, b.EPS), args.warmup, args.iters)
    fused_ms = time_ms(lambda: fused(x), args.warmup, args.iters)
    print(f"config={args.config} variant={args.variant}")
    print(f"gpu={torch.cuda.get_device_name(0)} dtype={dtype}")
    print(f"shape=({tokens}, {hidden}) -> {out}")
    print(f"max_abs_diff={float(diff.max()):.6e}")
    print(f"mean_abs_diff={float(diff.mean()):.6e}")
    print(f"baseline_ms={baseline_ms:.4f}")
    print(f"fused_ms={fused_ms:.4f}")
    print(f"speedup={baseline_ms / fused_ms:.3f}x")
    print(f"fused_tflops={b.flops_of(tokens, hidden, out) / (fused_ms * 1e-3) / 1e12:.1f}")


if __name__ == "__main__":
    main()
