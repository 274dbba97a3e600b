"""CPU oracle for the fused RMSNorm -> Linear path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product (the library, the
``denominator_cuda`` module, the ``src`` package) imports this file; only
tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline / reference
arm use it, and only as the checker or the CPU baseline.

Each function restates, with torch CPU ops, one step of the reference's own
unfused path or of its int8 quantization-aware path:

* simple_rmsnorm          - src/benchmark_kimi26.py:23-31 (SimpleRMSNorm.forward)
* unfused_reference       - src/benchmark_kimi26.py:94 (linear(norm(x)))
* fold_gamma              - src/weight_transform.py:104 (W_new = W * gamma)
* quantize_int8_per_output_channel - src/benchmark_kimi26_quantized.py:30-35
* dequantize_int8         - src/benchmark_kimi26_quantized.py:38-39
* fused_quantized         - src/benchmark_kimi26_quantized.py:102-106
* fp32_truth / fp64_truth - the exact math the fused kernel approximates
* swiglu_normalize_reference - csrc/denominator_kernel.cu:1286-1369 (rmsnorm_swiglu)
* swiglu_module_reference - src/fused_forward.py:274-284 (FusedRMSNormSwiGLUV1.forward)
* swiglu_unfused_reference - the model's silu(gate(norm(x))) * up(norm(x))

The restatement is pinned against outputs of the reference itself, generated
in the build container by tests/golden/make_golden.py and committed as
tests/golden/*.npz (checked by tests/test_oracle_golden.py).
"""

from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

# ----------------------------------------------------------- reference path


def simple_rmsnorm(x: torch.Tensor, gamma: torch.Tensor, eps: float) -> torch.Tensor:
    """x * bf16(rsqrt(mean(f32(x)^2) + eps)) * bf16(gamma), in x's dtype.

    Two roundings to x's dtype, exactly as SimpleRMSNorm.forward: the fp32
    inverse RMS is cast to x's dtype before the multiply, and gamma is cast to
    x's dtype (reference src/benchmark_kimi26.py:29-31).
    """
    variance = x.float().pow(2).mean(dim=-1, keepdim=True)
    return x * torch.rsqrt(variance + eps).to(x.dtype) * gamma.to(x.dtype)


def torch_rmsnorm(x: torch.Tensor, gamma: torch.Tensor, eps: float) -> torch.Tensor:
    """torch.nn.RMSNorm semantics (the Llama decode sweep's norm,
    reference src/benchmark.py:1008): normalise in fp32 math, scale by gamma."""
    return F.rms_norm(x, (x.shape[-1],), gamma.to(x.dtype), eps)


def unfused_reference(x: torch.Tensor, gamma: torch.Tensor, W: torch.Tensor,
                      b: torch.Tensor | None, eps: float, norm: str = "simple") -> torch.Tensor:
    """linear(norm(x)) on the CPU in x's dtype (bf16 matmul accumulates fp32)."""
    y = simple_rmsnorm(x, gamma, eps) if norm == "simple" else torch_rmsnorm(x, gamma, eps)
    return F.linear(y, W, b)


def fold_gamma(W: torch.Tensor, gamma: torch.Tensor) -> torch.Tensor:
    """W * gamma with torch's broadcasting and W's rounding."""
    return W * gamma


def fp32_truth(x: torch.Tensor, W_fused: torch.Tensor, b: torch.Tensor | None,
               eps: float) -> torch.Tensor:
    """inv_rms[m] * (x . W_fused^T) + b with fp32 inputs and fp32 math: what
    the fused kernel computes before its single rounding."""
    xf = x.float()
    inv_rms = torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + eps)
    out = (xf @ W_fused.float().t()) * inv_rms
    if b is not None:
        out = out + b.float()
    return out


def fp64_truth(x: np.ndarray, W_fused: np.ndarray, b: np.ndarray | None,
               eps: float) -> np.ndarray:
    """The same math in numpy float64 (independent of torch's kernels)."""
    xd = x.astype(np.float64)
    inv_rms = 1.0 / np.sqrt((xd * xd).mean(axis=-1, keepdims=True) + eps)
    out = (xd @ W_fused.astype(np.float64).T) * inv_rms
    if b is not None:
        out = out + b.astype(np.float64)
    return out


def inv_rms(x: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    return torch.rsqrt(xf.pow(2).mean(dim=-1) + eps)


def normalize_inplace_reference(x: torch.Tensor, raw: torch.Tensor, b: torch.Tensor,
                                eps: float) -> torch.Tensor:
    """What rmsnorm_normalize(_512) writes: round(raw * inv_rms + b), fp32 math
    (reference csrc/denominator_kernel.cu:1202-1273)."""
    r = inv_rms(x, eps)
    return (raw.float() * r[:, None] + b.float()).to(raw.dtype)


# ------------------------------------------------------------- SwiGLU path


def swiglu_normalize_reference(x: torch.Tensor, raw: torch.Tensor, b: torch.Tensor,
                               intermediate: int, eps: float) -> torch.Tensor:
    """What rmsnorm_swiglu(_512) writes from a [gate | up] GEMM output, fp32 math
    and one rounding (reference csrc/denominator_kernel.cu:1286-1369):
    g = raw[:, :I] * inv_rms + b[:I], u = raw[:, I:] * inv_rms + b[I:],
    out = g / (1 + exp(-g)) * u."""
    r = inv_rms(x, eps)[:, None]
    rf, bf = raw.float(), b.float()
    g = rf[:, :intermediate] * r + bf[:intermediate]
    u = rf[:, intermediate:] * r + bf[intermediate:]
    return (g / (1.0 + torch.exp(-g)) * u).to(raw.dtype)


def swiglu_module_reference(x: torch.Tensor, W_combined: torch.Tensor, b: torch.Tensor,
                            intermediate: int, eps: float) -> torch.Tensor:
    """FusedRMSNormSwiGLUV1/V3.forward of the reference: F.linear(x,
    W_combined) rounded to x's dtype, then rmsnorm_swiglu
    (reference src/fused_forward.py:274-284)."""
    return swiglu_normalize_reference(x, F.linear(x, W_combined), b, intermediate, eps)


def swiglu_unfused_reference(x: torch.Tensor, gamma: torch.Tensor, W_gate: torch.Tensor,
                             W_up: torch.Tensor, eps: float, norm: str = "torch") -> torch.Tensor:
    """The model's own MLP input: silu(gate_proj(norm(x))) * up_proj(norm(x)) in
    x's dtype (Llama's post_attention_layernorm -> act_fn(gate) * up)."""
    y = simple_rmsnorm(x, gamma, eps) if norm == "simple" else torch_rmsnorm(x, gamma, eps)
    return F.silu(F.linear(y, W_gate)) * F.linear(y, W_up)


def swiglu_fp32_truth(x: torch.Tensor, W_combined: torch.Tensor, b: torch.Tensor | None,
                      intermediate: int, eps: float) -> torch.Tensor:
    """silu(inv_rms * x.Wg^T + b_g) * (inv_rms * x.Wu^T + b_u) in fp32: the fused
    SwiGLU kernel's math before its single rounding."""
    gu = fp32_truth(x, W_combined, b, eps)
    g, u = gu[:, :intermediate], gu[:, intermediate:]
    return g / (1.0 + torch.exp(-g)) * u


# ----------------------------------------------------------------- int8 path


def quantize_int8_per_output_channel(weight: torch.Tensor):
    """Symmetric per-row int8: scale = max(|w|, 1e-8) / 127, q = clamp(round(w /
    scale), -127, 127).  Returns (q int8 [N, K], scale fp32 [N])."""
    w = weight.float()
    scale = w.abs().amax(dim=1, keepdim=True).clamp_min(1e-8) / 127.0
    q = torch.round(w / scale).clamp(-127, 127).to(torch.int8)
    return q, scale.squeeze(1)


def dequantize_int8(qweight: torch.Tensor, scale: torch.Tensor, dtype: torch.dtype):
    return (qweight.float() * scale.float().unsqueeze(1)).to(dtype)


def fused_quantized(x: torch.Tensor, qweight: torch.Tensor, scale: torch.Tensor, eps: float,
                    dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """F.linear(x * bf16(inv_rms), dequantized W): the reference's fused
    quantization-aware forward."""
    w = dequantize_int8(qweight, scale, dtype)
    variance = x.float().pow(2).mean(dim=-1, keepdim=True)
    r = torch.rsqrt(variance + eps).to(dtype)
    return F.linear(x * r, w)


def int8_fp32_truth(x: torch.Tensor, qweight: torch.Tensor, scale: torch.Tensor,
                    b: torch.Tensor | None, eps: float) -> torch.Tensor:
    """inv_rms[m] * scale[n] * (x . q^T) + b in fp32: the int8 kernel's math."""
    xf = x.float()
    r = torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + eps)
    out = (xf @ qweight.float().t()) * r * scale.float()[None, :]
    if b is not None:
        out = out + b.float()
    return out


# ------------------------------------------------------------ seeded inputs

# Workload shapes: (tokens M, hidden K, out N).
CONFIGS = {
    "kimi_q_b": (512, 1536, 12288),
    "kimi_kv_b": (512, 512, 16384),
    "kimi_q_b_long": (4096, 1536, 12288),
    "kimi_kv_b_long": (4096, 512, 16384),
    "decode_m1": (1, 4096, 6144),
    "decode_m8": (8, 4096, 6144),
    "decode_m32": (32, 4096, 6144),
    "decode_m128": (128, 4096, 6144),
    "int8_q_b": (2048, 1536, 12288),
}
EPS = 1e-5


def make_inputs(M: int, K: int, N: int, seed: int = 1234, dtype=torch.bfloat16,
                device="cpu"):
    """x ~ N(0,1) [M,K], gamma ~ 1 + 0.1 N(0,1) [K], W ~ N(0, 1/K) [N,K].

    Drawn in fp32 from one seeded generator (x, then gamma, then W) and
    rounded to `dtype`, so every consumer sees the same bits.
    """
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = torch.randn(M, K, generator=g, dtype=torch.float32)
    gamma = 1.0 + 0.1 * torch.randn(K, generator=g, dtype=torch.float32)
    W = torch.randn(N, K, generator=g, dtype=torch.float32) / np.sqrt(K)
    return x.to(dtype).to(device), gamma.to(dtype).to(device), W.to(dtype).to(device)


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def from_bf16_bits(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)
