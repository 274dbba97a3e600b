"""Decode-step grouped-query attention modules (reference
src/gqa_attention_forward.py): ``GQADecodeAttentionV2`` and
``GQADecodeAttentionV3`` with the reference's constructor and forward
signatures, and ``pytorch_gqa_decode_attention``, the reference's plain
PyTorch formulation that its tests compare against.

Both module variants run the same sm_100a kernel (context split across SMs,
one K/V read per KV head for its whole query group); V2 / V3 differ only in
which reference export they mirror.
"""

from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from src.load_gqa_attention import gqa_attention_cuda


class GQADecodeAttentionV2(nn.Module):
    """q [batch, Hq, D], k_cache / v_cache [batch, ctx, Hkv, D] -> [batch, Hq, D]."""

    def __init__(self, num_q_heads, num_kv_heads, head_dim):
        super().__init__()
        self.num_q_heads = num_q_heads
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.scale = 1.0 / math.sqrt(head_dim)

    def forward(self, q, k_cache, v_cache):
        output = torch.empty_like(q)
        gqa_attention_cuda.gqa_decode_v2(q, k_cache, v_cache, output, self.scale)
        return output


class GQADecodeAttentionV3(nn.Module):
    """As V2, with the group size passed explicitly (reference V3)."""

    def __init__(self, num_q_heads, num_kv_heads, head_dim):
        super().__init__()
        self.num_q_heads = num_q_heads
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.group_size = num_q_heads // num_kv_heads
        self.scale = 1.0 / math.sqrt(head_dim)

    def forward(self, q, k_cache, v_cache):
        output = torch.empty_like(q)
        gqa_attention_cuda.gqa_decode_v3(q, k_cache, v_cache, output, self.group_size,
                                         self.scale)
        return output


def pytorch_gqa_decode_attention(q, k_cache, v_cache, num_kv_heads):
    """Plain PyTorch decode attention (the reference's comparison path):
    repeat each KV head over its query group and run SDPA."""
    batch, num_q_heads, head_dim = q.shape
    group_size = num_q_heads // num_kv_heads
    scale = 1.0 / math.sqrt(head_dim)
    k = k_cache.repeat_interleave(group_size, dim=2).permute(0, 2, 1, 3)
    v = v_cache.repeat_interleave(group_size, dim=2).permute(0, 2, 1, 3)
    out = F.scaled_dot_product_attention(q.unsqueeze(2), k, v, scale=scale)
    return out.squeeze(2)
