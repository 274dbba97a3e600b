"""Quantization-aware Kimi benchmark (same CLI and output lines as the
reference's src/benchmark_kimi26_quantized.py:42-126), with the fused path
running the int8-weight kernel instead of dequantize-then-F.linear.

    python -m src.benchmark_kimi26_quantized --config kimi_q_b --tokens 2048
"""

from __future__ import annotations

import argparse

import torch
import torch.nn as nn
import torch.nn.functional as F

from src.benchmark_kimi26 import CONFIGS, SimpleRMSNorm, bench
from src.quantized import FusedRMSNormLinearInt8, dequantize_int8, quantize_int8_per_output_channel
from src.weight_transform import compute_fused_weights_rmsnorm


def parse_args(argv=None) -> argparse.Namespace:
    p = argparse.ArgumentParser(description="Benchmark int8-weight fused RMSNorm+Linear on B200.")
    p.add_argument("--config", choices=CONFIGS.keys(), default="kimi_q_b")
    p.add_argument("--tokens", type=int)
    p.add_argument("--hidden", type=int)
    p.add_argument("--out", type=int)
    p.add_argument("--dtype", choices=["bfloat16", "float16"], default="bfloat16")
    p.add_argument("--warmup", type=int, default=30)
    p.add_argument("--iters", type=int, default=300)
    p.add_argument("--cuda-events", action="store_true")
    return p.parse_args(argv)


def main(argv=None) -> None:
    if not torch.cuda.is_available():
        raise SystemExit("CUDA is required.")
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
    q_w, q_scale = quantize_int8_per_output_channel(linear.weight.detach())

    W_new, b_new, h, eps = compute_fused_weights_rmsnorm(norm, linear)
    fused = FusedRMSNormLinearInt8(W_new, b_new, h, eps)

    def baseline_quantized(t):
        return F.linear(norm(t), dequantize_int8(q_w, q_scale, dtype))

    def reference_fused_quantized(t):
        w = dequantize_int8(fused.qweight, fused.w_scale, dtype)
        variance = t.float().pow(2).mean(dim=-1, keepdim=True)
        return F.linear(t * torch.rsqrt(variance + eps).to(dtype), w)

    with torch.no_grad():
        diff = (baseline_quantized(x).float() - fused(x).float()).abs()
        diff_ref = (reference_fused_quantized(x).float() - fused(x).float()).abs()
    baseline_ms = bench(baseline_quantized, x, args.warmup, args.iters, args.cuda_events)
    ref_fused_ms = bench(reference_fused_quantized, x, args.warmup, args.iters, args.cuda_events)
    fused_ms = bench(fused, x, args.warmup, args.iters, args.cuda_events)
    print(f"config={args.config} quantization=int8_per_output_channel")
    print(f"gpu={torch.cuda.get_device_name(0)} dtype={dtype}")
    print(f"shape=({tokens}, {hidden}) -> {out}")
    print("note=int8 weights are widened to bf16 inside the GEMM mainloop")
    print(f"max_abs_diff={float(diff.max()):.6e}")
    print(f"mean_abs_diff={float(diff.mean()):.6e}")
    print(f"max_abs_diff_vs_reference_fused={float(diff_ref.max()):.6e}")
    print(f"baseline_quantized_ms={baseline_ms:.4f}")
    print(f"reference_fused_quantized_ms={ref_fused_ms:.4f}")
    print(f"fused_quantized_ms={fused_ms:.4f}")
    print(f"speedup={baseline_ms / fused_ms:.3f}x")


if __name__ == "__main__":
    main()
