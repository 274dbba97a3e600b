"""Swap Kimi K2.6 / DeepseekV3 attention LoRA norm pairs for the fused op.

Inside each decoder layer's ``self_attn`` the attention code computes

    q_b_proj(q_a_layernorm(...))        kv_b_proj(kv_a_layernorm(k_pass))

For each pair this module replaces the Linear with a fused RMSNorm -> Linear
module built from the gamma-folded weight and the norm with an identity
marker, leaving the model's own forward untouched.  The public function,
its arguments, return value, count keys and the marker class name match the
reference (src/patch_kimi.py:29-148), so the resulting module tree and
state_dict keys are the same (``...q_b_proj.W_new``, ``...q_b_proj.b_new``;
the norms' ``weight`` entries disappear).

The main input/post-attention norms are left alone: they feed RoPE, the KV
cache and MoE routing, not a single Linear.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from src.fused_forward import FusedRMSNormLinearV1, FusedRMSNormLinearV3
from src.quantized import FusedRMSNormLinearInt8
from src.weight_transform import compute_fused_weights_rmsnorm

# "V1"/"V3" as in the reference; "INT8" quantizes the folded weight per output
# channel and runs the int8-weight fused kernel.
_VARIANT_CLASSES = {
    "V1": FusedRMSNormLinearV1,
    "V3": FusedRMSNormLinearV3,
    "INT8": FusedRMSNormLinearInt8,
}

# (norm attribute, linear attribute, count key) of the pairs this patch fuses.
_PAIRS = (
    ("q_a_layernorm", "q_b_proj", "q_a_layernorm_to_q_b_proj"),
    ("kv_a_layernorm", "kv_b_proj", "kv_a_layernorm_to_kv_b_proj"),
)

# Attribute paths under which HF wrappers keep the decoder layer list.
_LAYER_PATHS = (
    ("model", "layers"),
    ("language_model", "model", "layers"),
    ("language_model", "layers"),
    ("text_model", "layers"),
    ("model", "model", "layers"),
)


class _AlreadyPatchedIdentity(nn.Identity):
    """Identity left in place of a folded norm; marks the pair as done so a
    second patch call skips it."""


def _resolve_text_layers(model) -> list[nn.Module]:
    """Return the decoder layers of a Kimi / DeepseekV3 model or wrapper."""
    for path in _LAYER_PATHS:
        node = model
        for attr in path:
            node = getattr(node, attr, None)
            if node is None:
                break
        if isinstance(node, (list, nn.ModuleList)):
            return list(node)
    raise AttributeError(
        "Could not find Kimi decoder layers. Inspect model.named_modules() and "
        "update _resolve_text_layers for this model wrapper.")


def _patch_norm_linear_pair(owner: nn.Module, norm_name: str, linear_name: str, *,
                            device: torch.device, variant: str) -> bool:
    """Fuse ``owner.<norm_name>`` into ``owner.<linear_name>``; False if the
    pair is missing, already patched, or not (norm with weight, nn.Linear)."""
    norm = getattr(owner, norm_name, None)
    linear = getattr(owner, linear_name, None)
    if norm is None or linear is None or isinstance(norm, _AlreadyPatchedIdentity):
        return False
    if not hasattr(norm, "weight") or not isinstance(linear, nn.Linear):
        return False
    W_new, b_new, h, eps = compute_fused_weights_rmsnorm(norm, linear)
    fused = _VARIANT_CLASSES[variant](W_new.to(device), b_new.to(device), h, eps)
    setattr(owner, linear_name, fused)
    setattr(owner, norm_name, _AlreadyPatchedIdentity())
    return True


def patch_kimi_q_lora_norms(model, device=None, variant: str = "V3") -> dict[str, int]:
    """Patch every layer's q_a/kv_a LoRA RMSNorm -> projection pair in place.

    Args:
        model: Kimi K2.6 (DeepseekV3-style) HF model or its text model.
        device: where the fused weights live; default: the model's first
            parameter's device.
        variant: "V1" or "V3" (both run the same sm_100a fused kernel), or
            "INT8" for int8 per-channel weights.

    Returns:
        ``{"q_a_layernorm_to_q_b_proj": n_q, "kv_a_layernorm_to_kv_b_proj": n_kv}``.
    """
    if variant not in _VARIANT_CLASSES:
        raise ValueError(f"Unknown variant {variant!r}; choose from {list(_VARIANT_CLASSES)}")
    if device is None:
        device = next(model.parameters()).device
    counts = {key: 0 for _, _, key in _PAIRS}
    for layer in _resolve_text_layers(model):
        attn = getattr(layer, "self_attn", None)
        if attn is None:
            continue
        for norm_name, linear_name, key in _PAIRS:
            if _patch_norm_linear_pair(attn, norm_name, linear_name, device=device,
                                       variant=variant):
                counts[key] += 1
    return counts


def print_kimi_patchable_pairs(model) -> None:
    """Print, per layer, which fusable norm -> projection pairs it has."""
    for idx, layer in enumerate(_resolve_text_layers(model)):
        attn = getattr(layer, "self_attn", None)
        if attn is None:
            continue
        found = [f"{n} -> {l}" for n, l, _ in _PAIRS if hasattr(attn, n) and hasattr(attn, l)]
        if found:
            print(f"layer {idx}: " + ", ".join(found))
