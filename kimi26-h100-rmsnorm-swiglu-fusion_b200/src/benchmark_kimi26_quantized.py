"""Quantization-aware Kimi benchmark with the reference's command line and
key=value lines (reference src/benchmark_kimi26_quantized.py:42-126), the
fused path running this library's int8-weight kernel instead of
dequantize-then-F.linear:

    python -m src.benchmark_kimi26_quantized --config kimi_q_b --tokens 2048

Inputs and timing come from the repository's bench.py (through
src.benchmark_kimi26): the baseline is the reference's unfused quantized path
(W quantized before gamma folding, norm then F.linear over the dequantized
weight), its fused quantized path dequantizes W_fused and scales x by
bf16(inv_rms); the int8 kernel is timed through FusedRMSNormLinearInt8.
"""

from __future__ import annotations

import argparse

import torch
import torch.nn.functional as F

from src.benchmark_kimi26 import CONFIGS, bench_module, shape_of, time_ms
from src.quantized import FusedRMSNormLinearInt8, dequantize_int8, quantize_int8_per_output_channel


def parse_args(argv=None) -> argparse.Namespace:
    p = argparse.ArgumentParser(description="Benchmark int8-weight fused RMSNorm+Linear on B200.")
    p.add_argument("--config", choices=CONFIGS.keys(), default="kimi_q_b")
    p.add_argument("--tokens", type=int)
    p.add_argument("--hidden", type=int)
    p.add_argument("--out", type=int)
    p.add_argument("--dtype", choices=["bfloat16", "float16"], default="bfloat16")
    p.add_argument("--warmup", type=int, default=30)
    p.add_argument("--iters", type=int, default=300)
    return p.parse_args(argv)


def main(argv=None) -> None:
    if not torch.cuda.is_available():
        raise SystemExit("CUDA is required.")
    args = parse_args(argv)
    dtype = getattr(torch, args.dtype)
    tokens, hidden, out = shape_of(args)
    b = bench_module()
    x, gamma, W = (t.to(dtype) for t in b.gpu_inputs(tokens, hidden, out, 1234, "cuda"))
    eps = b.EPS
    q_w, q_scale = quantize_int8_per_output_channel(W)             # before folding
    W_new = W * gamma
    fused = FusedRMSNormLinearInt8(W_new, torch.zeros(out, dtype=dtype, device="cuda"),
                                   hidden, eps)                      # after folding

    def norm(t):
        r = torch.rsqrt(t.float().pow(2).mean(dim=-1, keepdim=True) + eps)
        return t * r.to(dtype) * gamma

    def baseline_quantized():
        return F.linear(norm(x), dequantize_int8(q_w, q_scale, dtype))

    def reference_fused_quantized():
        r = torch.rsqrt(x.float().pow(2).mean(dim=-1, keepdim=True) + eps)
        return F.linear(x * r.to(dtype), dequantize_int8(fused.qweight, fused.w_scale, dtype))

    with torch.no_grad():
        ours = fused(x).float()
        diff = (baseline_quantized().float() - ours).abs()
        diff_ref = (reference_fused_quantized().float() - ours).abs()
    baseline_ms = time_ms(baseline_quantized, args.warmup, args.iters)
    ref_fused_ms = time_ms(reference_fused_quantized, args.warmup, args.iters)
    fused_ms = time_ms(lambda: fused(x), args.warmup, args.iters)
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
