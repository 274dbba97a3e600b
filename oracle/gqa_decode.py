"""CPU oracle for decode-step grouped-query attention.

TEST INFRASTRUCTURE ONLY (see oracle/rmsnorm_linear.py).  Restates, in fp64
numpy, what the reference's gqa_decode_v2 / gqa_decode_v3 kernels compute
(csrc/gqa_attention_kernel.cu:76-350: per query head h, scores
scale * q[h] . K[t, h // G], an online softmax over the context, weights
applied to V[t, h // G]) and what its PyTorch comparison path computes
(src/gqa_attention_forward.py:76-110, SDPA over repeated KV heads).
"""

from __future__ import annotations

import numpy as np
import torch


def gqa_decode_reference(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                         scale: float) -> torch.Tensor:
    """q [B, Hq, D], caches [B, T, Hkv, D] -> out [B, Hq, D] in fp32 (fp64 math)."""
    qd = q.double().numpy()
    kd = k_cache.double().numpy()
    vd = v_cache.double().numpy()
    B, Hq, D = qd.shape
    Hkv = kd.shape[2]
    G = Hq // Hkv
    out = np.empty((B, Hq, D))
    for h in range(Hq):
        kh = kd[:, :, h // G, :]                        # [B, T, D]
        vh = vd[:, :, h // G, :]
        s = np.einsum("bd,btd->bt", qd[:, h, :], kh) * scale
        s -= s.max(axis=1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(axis=1, keepdims=True)
        out[:, h, :] = np.einsum("bt,btd->bd", p, vh)
    return torch.from_numpy(out).float()


def make_gqa_inputs(B, Hq, Hkv, D, T, seed=0, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, Hq, D, generator=g)
    k = torch.randn(B, T, Hkv, D, generator=g)
    v = torch.randn(B, T, Hkv, D, generator=g)
    return q.to(dtype), k.to(dtype), v.to(dtype)
