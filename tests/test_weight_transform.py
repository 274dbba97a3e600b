"""The product's gamma folding is bit-identical to the reference's
(golden vectors from the reference's compute_fused_weights_rmsnorm*)."""
import os

import numpy as np
import pytest
import torch
import torch.nn as nn

from oracle import rmsnorm_linear as orc
from src import weight_transform as wt

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "golden_cases.npz")
CASES = ["q_b_small", "kv_b_small", "decode_small", "ragged_bias", "tall_bias"]


class _VarEpsNorm(nn.Module):
    """HF-style norm that names its epsilon variance_epsilon."""

    def __init__(self, gamma, eps):
        super().__init__()
        self.weight = nn.Parameter(gamma.clone())
        self.variance_epsilon = eps


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


@pytest.mark.parametrize("name", CASES)
@pytest.mark.parametrize("norm_kind", ["variance_epsilon", "torch"])
def test_compute_fused_weights_rmsnorm_bits(golden, name, norm_kind):
    M, K, N = (int(v) for v in golden[f"{name}__shape"])
    gamma = orc.from_bf16_bits(golden[f"{name}__gamma"])
    W = orc.from_bf16_bits(golden[f"{name}__W"]).reshape(N, K)
    has_bias = bool(golden[f"{name}__has_bias"][0])
    b = orc.from_bf16_bits(golden[f"{name}__b"])
    if norm_kind == "torch":
        norm = nn.RMSNorm(K, eps=1e-5).to(torch.bfloat16)
        with torch.no_grad():
            norm.weight.copy_(gamma)
        key = f"{name}__W_new_torchnorm"
    else:
        norm = _VarEpsNorm(gamma, 1e-5)
        key = f"{name}__W_new"
    lin = nn.Linear(K, N, bias=has_bias).to(torch.bfloat16)
    with torch.no_grad():
        lin.weight.copy_(W)
        if has_bias:
            lin.bias.copy_(b)
    W_new, b_new, h, eps = wt.compute_fused_weights_rmsnorm(norm, lin)
    want = orc.from_bf16_bits(golden[key]).reshape(N, K)
    assert torch.equal(W_new.view(torch.int16), want.view(torch.int16))
    assert h == K and eps == 1e-5
    assert b_new.dtype == W.dtype and b_new.shape == (N,)
    if has_bias:
        assert torch.equal(b_new.view(torch.int16), b.view(torch.int16))
    else:
        assert torch.count_nonzero(b_new) == 0


def test_combined_bits(golden):
    gamma = orc.from_bf16_bits(golden["combined__gamma"])
    norm = nn.RMSNorm(64, eps=1e-5).to(torch.bfloat16)
    with torch.no_grad():
        norm.weight.copy_(gamma)
    lins = []
    for i in range(3):
        W = orc.from_bf16_bits(golden[f"combined__W{i}"]).reshape(-1, 64)
        lin = nn.Linear(64, W.shape[0], bias=False).to(torch.bfloat16)
        with torch.no_grad():
            lin.weight.copy_(W)
        lins.append(lin)
    Wc, bc, splits, h, eps = wt.compute_fused_weights_rmsnorm_combined(norm, lins)
    want = orc.from_bf16_bits(golden["combined__W_combined"]).reshape(-1, 64)
    assert torch.equal(Wc.view(torch.int16), want.view(torch.int16))
    assert splits == [64, 16, 16] and h == 64 and eps == 1e-5
    assert bc.shape == (96,) and torch.count_nonzero(bc) == 0


def test_eps_none_resolves_like_torch_rmsnorm():
    norm = nn.RMSNorm(16, eps=None)
    lin = nn.Linear(16, 8, bias=False)
    _, _, _, eps = wt.compute_fused_weights_rmsnorm(norm, lin)
    assert eps == torch.finfo(torch.float32).eps


def test_llama_layer_transforms():
    from transformers import LlamaConfig
    from transformers.models.llama.modeling_llama import LlamaDecoderLayer

    cfg = LlamaConfig(hidden_size=64, intermediate_size=96, num_attention_heads=4,
                      num_key_value_heads=2, rms_norm_eps=1e-5)
    torch.manual_seed(0)
    layer = LlamaDecoderLayer(cfg, layer_idx=0)
    sep = wt.transform_llama_layer(layer)
    assert set(sep) == {"attn_q_proj", "attn_k_proj", "attn_v_proj", "gate_proj", "up_proj"}
    comb = wt.transform_llama_layer_combined(layer)
    Wqkv, bqkv, splits, h, eps = comb["attn_qkv"]
    assert splits == [64, 32, 32] and h == 64 and eps == 1e-5
    assert torch.equal(Wqkv[:64], sep["attn_q_proj"][0])
    Wgu, _, gsplits, _, _ = comb["mlp_gate_up"]
    assert gsplits == [96, 96] and torch.equal(Wgu[96:], sep["up_proj"][0])
