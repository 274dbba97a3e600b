"""Patch a Llama model (HF ``LlamaForCausalLM``) to run its norm -> projection
pairs through the fused RMSNorm kernels.

Same entry point, arguments and attached module names as the reference
(src/patch_llama.py:47-90): per decoder layer

* separate (default): ``self_attn.fused_{q,k,v}_proj`` under input_layernorm
  and ``mlp.fused_{gate,up}_proj`` under post_attention_layernorm;
* ``combined=True``: ``self_attn.fused_qkv`` (one launch whose Q/K/V parts
  are written straight into their own tensors) and ``mlp.fused_gate_up``;
* ``swiglu=True`` (implies combined): ``mlp.fused_gate_up_swiglu``, one launch
  for norm -> gate/up -> silu(gate) * up;
* ``gqa_decode=True``: ``self_attn.gqa_decode_module`` (GQADecodeAttentionV3)
  takes single-token decode steps when the model has fewer KV than Q heads.

The layer and attention forwards are replaced by ones that skip the two
RMSNorm calls (their gamma is folded into the fused weights and their
1/rms is applied inside the kernels) and are otherwise the installed
transformers' own LlamaDecoderLayer / LlamaAttention forwards.  The original
projections stay on the module, as in the reference.  down_proj follows an
activation, not a norm, and is not fused.
"""

from __future__ import annotations

from typing import Callable

import torch
from transformers.models.llama.modeling_llama import (
    ALL_ATTENTION_FUNCTIONS,
    apply_rotary_pos_emb,
    eager_attention_forward,
)

from src.fused_forward import (
    FusedRMSNormCombinedLinearV1,
    FusedRMSNormCombinedLinearV3,
    FusedRMSNormLinearV1,
    FusedRMSNormLinearV3,
    FusedRMSNormSwiGLUV1,
    FusedRMSNormSwiGLUV3,
)
from src.gqa_attention_forward import GQADecodeAttentionV3
from src.weight_transform import transform_llama_layer, transform_llama_layer_combined

_VARIANT_CLASSES = {"V1": FusedRMSNormLinearV1, "V3": FusedRMSNormLinearV3}
_COMBINED_VARIANT_CLASSES = {"V1": FusedRMSNormCombinedLinearV1,
                             "V3": FusedRMSNormCombinedLinearV3}
_SWIGLU_VARIANT_CLASSES = {"V1": FusedRMSNormSwiGLUV1, "V3": FusedRMSNormSwiGLUV3}


def patch_llama_model(model, device=None, variant="V1", combined=False, swiglu=False,
                      gqa_decode=False):
    """Patch every decoder layer of a Llama model in place; returns the model.

    variant: "V1" or "V3" (both run the same sm_100a kernels); combined: one
    fused launch for Q/K/V and one for gate/up; swiglu (implies combined):
    gate/up and the SiLU product in one launch; gqa_decode: custom decode
    attention for single-token steps of a GQA model.
    """
    if variant not in _VARIANT_CLASSES:
        raise ValueError(f"Unknown variant {variant!r}; choose from {list(_VARIANT_CLASSES)}")
    if swiglu:
        combined = True
    if device is None:
        device = next(model.parameters()).device
    config = model.config
    num_q_heads = config.num_attention_heads
    num_kv_heads = config.num_key_value_heads
    head_dim = getattr(config, "head_dim", None) or config.hidden_size // num_q_heads

    for layer in model.model.layers:
        if swiglu:
            _patch_decoder_layer_swiglu(layer, device, variant)
        elif combined:
            _patch_decoder_layer_combined(layer, device, variant)
        else:
            _patch_decoder_layer(layer, device, variant)
        if gqa_decode and num_kv_heads < num_q_heads:
            layer.self_attn.gqa_decode_module = GQADecodeAttentionV3(num_q_heads, num_kv_heads,
                                                                     head_dim)
    return model


# ------------------------------------------------------------ layer patchers


def _patch_decoder_layer(layer, device, variant="V1"):
    fused = transform_llama_layer(layer)
    cls = _VARIANT_CLASSES[variant]
    for name in ("q_proj", "k_proj", "v_proj"):
        W, b, h, eps = fused[f"attn_{name}"]
        setattr(layer.self_attn, f"fused_{name}", cls(W.to(device), b.to(device), h, eps))
    for name in ("gate_proj", "up_proj"):
        W, b, h, eps = fused[name]
        setattr(layer.mlp, f"fused_{name}", cls(W.to(device), b.to(device), h, eps))
    attn = layer.self_attn
    _patch_attention_forward(attn, lambda x: (attn.fused_q_proj(x), attn.fused_k_proj(x),
                                              attn.fused_v_proj(x)))
    mlp = layer.mlp
    _patch_layer_forward(layer, lambda x: mlp.down_proj(
        mlp.act_fn(mlp.fused_gate_proj(x)) * mlp.fused_up_proj(x)))


def _patch_decoder_layer_combined(layer, device, variant="V1"):
    fused = transform_llama_layer_combined(layer)
    cls = _COMBINED_VARIANT_CLASSES[variant]
    W, b, sizes, h, eps = fused["attn_qkv"]
    layer.self_attn.fused_qkv = cls(W.to(device), b.to(device), sizes, h, eps)
    W, b, sizes, h, eps = fused["mlp_gate_up"]
    layer.mlp.fused_gate_up = cls(W.to(device), b.to(device), sizes, h, eps)
    attn, mlp = layer.self_attn, layer.mlp
    _patch_attention_forward(attn, lambda x: tuple(attn.fused_qkv(x)))

    def mlp_forward(x):
        gate, up = mlp.fused_gate_up(x)
        return mlp.down_proj(mlp.act_fn(gate) * up)

    _patch_layer_forward(layer, mlp_forward)


def _patch_decoder_layer_swiglu(layer, device, variant="V1"):
    fused = transform_llama_layer_combined(layer)
    W, b, sizes, h, eps = fused["attn_qkv"]
    layer.self_attn.fused_qkv = _COMBINED_VARIANT_CLASSES[variant](
        W.to(device), b.to(device), sizes, h, eps)
    W, b, sizes, h, eps = fused["mlp_gate_up"]
    layer.mlp.fused_gate_up_swiglu = _SWIGLU_VARIANT_CLASSES[variant](
        W.to(device), b.to(device), sizes[0], h, eps)
    attn, mlp = layer.self_attn, layer.mlp
    _patch_attention_forward(attn, lambda x: tuple(attn.fused_qkv(x)))
    _patch_layer_forward(layer, lambda x: mlp.down_proj(mlp.fused_gate_up_swiglu(x)))


# ------------------------------------------------------------------ forwards


def _patch_attention_forward(attn, project_qkv: Callable):
    """LlamaAttention.forward with q/k/v from `project_qkv(raw hidden)` and
    the optional GQA decode path for single-token steps."""

    def forward(hidden_states: torch.Tensor, position_embeddings=None, attention_mask=None,
                past_key_values=None, **kwargs):
        input_shape = hidden_states.shape[:-1]
        hidden_shape = (*input_shape, -1, attn.head_dim)
        q, k, v = project_qkv(hidden_states)
        query_states = q.reshape(hidden_shape).transpose(1, 2)
        key_states = k.reshape(hidden_shape).transpose(1, 2)
        value_states = v.reshape(hidden_shape).transpose(1, 2)

        cos, sin = position_embeddings
        query_states, key_states = apply_rotary_pos_emb(query_states, key_states, cos, sin)
        if past_key_values is not None:
            key_states, value_states = past_key_values.update(key_states, value_states,
                                                              attn.layer_idx)

        if query_states.size(2) == 1 and hasattr(attn, "gqa_decode_module"):
            q_dec = query_states.squeeze(2).contiguous()          # [B, Hq, D]
            k_dec = key_states.permute(0, 2, 1, 3).contiguous()   # [B, T, Hkv, D]
            v_dec = value_states.permute(0, 2, 1, 3).contiguous()
            attn_output = attn.gqa_decode_module(q_dec, k_dec, v_dec).unsqueeze(2)
            attn_weights = None
        else:
            interface: Callable = ALL_ATTENTION_FUNCTIONS.get_interface(
                attn.config._attn_implementation, eager_attention_forward)
            attn_output, attn_weights = interface(
                attn, query_states, key_states, value_states, attention_mask,
                dropout=0.0 if not attn.training else attn.attention_dropout,
                scaling=attn.scaling, **kwargs)
        attn_output = attn_output.reshape(*input_shape, -1).contiguous()
        return attn.o_proj(attn_output), attn_weights

    attn.forward = forward


def _patch_layer_forward(layer, mlp_forward: Callable):
    """LlamaDecoderLayer.forward without the two RMSNorm calls."""

    def forward(hidden_states: torch.Tensor, attention_mask=None, position_ids=None,
                past_key_values=None, use_cache=False, position_embeddings=None, **kwargs):
        residual = hidden_states
        hidden_states, _ = layer.self_attn(
            hidden_states=hidden_states, attention_mask=attention_mask,
            position_ids=position_ids, past_key_values=past_key_values, use_cache=use_cache,
            position_embeddings=position_embeddings, **kwargs)
        hidden_states = residual + hidden_states
        residual = hidden_states
        return residual + mlp_forward(hidden_states)

    layer.forward = forward
