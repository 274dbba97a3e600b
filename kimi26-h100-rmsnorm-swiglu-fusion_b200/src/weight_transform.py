"""Offline gamma absorption for RMSNorm -> Linear pairs.

RMSNorm(x) = x * inv_rms(x) * gamma, so Linear(RMSNorm(x)) =
inv_rms(x) * (x @ (W * gamma)^T) + b.  Folding gamma into the weight once
(W_fused = W * gamma) leaves the forward pass one GEMM with a per-row scale,
which is what the fused kernel computes.

Function names, argument order and return tuples follow the reference
(src/weight_transform.py:69-109, :142-183, :186-212, :236-264) so that
patchers written against it run unchanged.  The product is formed with
torch's own broadcasting multiply in W's dtype, i.e. with the same rounding
as the reference, so the folded weights are bit-identical to its.
"""

from __future__ import annotations

import torch
import torch.nn as nn


def _norm_eps(rms_norm) -> float:
    """eps of an RMSNorm-like module: ``.eps`` if present, else
    ``.variance_epsilon`` (HF Llama/DeepseekV3 naming), as the reference
    reads it (src/weight_transform.py:100).  ``torch.nn.RMSNorm(eps=None)``
    means "finfo(dtype).eps"; that value is substituted so the fused op
    receives a number."""
    eps = rms_norm.eps if hasattr(rms_norm, "eps") else rms_norm.variance_epsilon
    if eps is None:
        eps = torch.finfo(rms_norm.weight.dtype).eps
    return eps


def _bias_or_zeros(linear: nn.Linear) -> torch.Tensor:
    W = linear.weight.data
    if linear.bias is not None:
        return linear.bias.data
    return torch.zeros(W.size(0), device=W.device, dtype=W.dtype)


def compute_fused_weights_rmsnorm(rms_norm, linear: nn.Linear):
    """Fold an RMSNorm's gamma into the following Linear.

    Returns ``(W_new, b_new, h, eps)``: ``W_new = W * gamma`` ([out, h], W's
    dtype), ``b_new`` the Linear's bias or zeros of W's dtype, ``h`` the
    normalised width and ``eps`` the norm's epsilon.
    """
    gamma = rms_norm.weight.data
    W = linear.weight.data
    W_new = W * gamma
    b_new = _bias_or_zeros(linear)
    return W_new, b_new, gamma.shape[0], _norm_eps(rms_norm)


def compute_fused_weights_rmsnorm_combined(rms_norm, linears):
    """Fold one RMSNorm into several Linears that share it (Q/K/V, gate/up).

    Returns ``(W_combined, b_combined, split_sizes, h, eps)`` with the folded
    weights and biases concatenated along the output dimension in the order
    given, and ``split_sizes`` the per-Linear output widths.
    """
    gamma = rms_norm.weight.data
    weights, biases, sizes = [], [], []
    for linear in linears:
        W = linear.weight.data
        weights.append(W * gamma)
        biases.append(_bias_or_zeros(linear))
        sizes.append(W.size(0))
    return (torch.cat(weights, dim=0), torch.cat(biases, dim=0), sizes, gamma.shape[0],
            _norm_eps(rms_norm))


def transform_llama_layer(decoder_layer) -> dict:
    """Per-projection folded weights of a Llama decoder layer.

    Keys ``attn_q_proj``, ``attn_k_proj``, ``attn_v_proj`` (input_layernorm)
    and ``gate_proj``, ``up_proj`` (post_attention_layernorm), each mapping to
    ``(W_new, b_new, h, eps)``.  down_proj follows an activation, not a norm,
    and is not folded.
    """
    attn, mlp = decoder_layer.self_attn, decoder_layer.mlp
    pre, post = decoder_layer.input_layernorm, decoder_layer.post_attention_layernorm
    fused = {}
    for name in ("q_proj", "k_proj", "v_proj"):
        fused[f"attn_{name}"] = compute_fused_weights_rmsnorm(pre, getattr(attn, name))
    for name in ("gate_proj", "up_proj"):
        fused[name] = compute_fused_weights_rmsnorm(post, getattr(mlp, name))
    return fused


def transform_llama_layer_combined(decoder_layer) -> dict:
    """Concatenated folded weights of a Llama decoder layer:
    ``attn_qkv`` (q, k, v under input_layernorm) and ``mlp_gate_up``
    (gate, up under post_attention_layernorm), each
    ``(W_combined, b_combined, split_sizes, h, eps)``."""
    attn, mlp = decoder_layer.self_attn, decoder_layer.mlp
    return {
        "attn_qkv": compute_fused_weights_rmsnorm_combined(
            decoder_layer.input_layernorm, [attn.q_proj, attn.k_proj, attn.v_proj]),
        "mlp_gate_up": compute_fused_weights_rmsnorm_combined(
            decoder_layer.post_attention_layernorm, [mlp.gate_proj, mlp.up_proj]),
    }


def transform_gpt_oss_layer(decoder_layer) -> dict:
    """``attn_qkv`` folded weights of a GPT-OSS layer (its MoE MLP sits behind
    a router and is not folded)."""
    attn = decoder_layer.self_attn
    return {"attn_qkv": compute_fused_weights_rmsnorm_combined(
        decoder_layer.input_layernorm, [attn.q_proj, attn.k_proj, attn.v_proj])}
