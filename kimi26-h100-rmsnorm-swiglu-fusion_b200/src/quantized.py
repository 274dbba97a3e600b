"""int8-weight fused RMSNorm -> Linear.

The reference studies weight-only int8 for the Kimi pairs with torch code
only (src/benchmark_kimi26_quantized.py): gamma is folded into W first, the
folded weight is quantized per output channel, and every call dequantizes the
whole weight to bf16 before F.linear(x * bf16(inv_rms), W_deq).  Here the
int8 bytes stay int8 in HBM and are widened inside the GEMM mainloop; inv_rms
and the per-channel scale are applied to the fp32 accumulator.

``quantize_int8_per_output_channel`` and ``dequantize_int8`` keep the
reference's names and numbers (torch ops, any device) for offline weight
preparation; the fused forward is ``FusedRMSNormLinearInt8``.
"""

from __future__ import annotations

import torch

from src.load_cuda import denominator_cuda


def quantize_int8_per_output_channel(weight: torch.Tensor):
    """Symmetric per-row int8: scale = max(|w|, 1e-8) / 127 (fp32),
    q = clamp(round(w / scale), -127, 127).  Returns (q int8, scale fp32 [N]).

    Same function and numbers as the reference
    (src/benchmark_kimi26_quantized.py:30-35).  On a CUDA tensor the sm_100a
    quantizer of this library produces bit-identical results."""
    if weight.is_cuda:
        return denominator_cuda.quantize_int8_per_channel(weight)
    w = weight.float()
    scale = w.abs().amax(dim=1, keepdim=True).clamp_min(1e-8) / 127.0
    q = torch.round(w / scale).clamp(-127, 127).to(torch.int8)
    return q, scale.squeeze(1)


def dequantize_int8(qweight: torch.Tensor, scale: torch.Tensor, dtype: torch.dtype):
    """(q * scale) rounded to `dtype` (reference src/benchmark_kimi26_quantized.py:38-39)."""
    return (qweight.float() * scale.float().unsqueeze(1)).to(dtype)


class FusedRMSNormLinearInt8(torch.nn.Module):
    """RMSNorm (gamma folded) -> Linear with an int8 per-channel weight.

    Built from the same (W_new, b_new, h, eps) as FusedRMSNormLinearV1/V3, so
    it can stand in for them in a patcher; W_new is quantized once at
    construction.  Buffers: ``qweight`` int8 [N, K], ``w_scale`` fp32 [N],
    ``b_new``."""

    def __init__(self, W_new: torch.Tensor, b_new: torch.Tensor, h: int, eps: float):
        super().__init__()
        q, scale = quantize_int8_per_output_channel(W_new)
        self.register_buffer("qweight", q)
        self.register_buffer("w_scale", scale.float())
        self.register_buffer("b_new", b_new)
        self.h = h
        self.eps = eps

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        orig_shape = x.shape
        if x.size(-1) != self.h:
            raise ValueError(f"x has {x.size(-1)} features but the module was built for h={self.h}")
        x_2d = x.reshape(-1, x.size(-1))
        out = denominator_cuda.fused_rmsnorm_linear_w8(x_2d, self.qweight, self.w_scale,
                                                       self.b_new, float(self.eps))
        return out.reshape(orig_shape[:-1] + (out.size(-1),))

    def extra_repr(self) -> str:
        return f"in={self.h}, out={self.qweight.shape[0]}, eps={self.eps}, int8 weights"
