"""patch_llama on a tiny random-init Llama (bf16, GQA 8 Q heads over 2 KV
heads, head_dim 64) on the GPU: logits of the patched model (separate,
combined, SwiGLU modes, and the GQA decode path for a cached single-token
step) against the unpatched model's own forward."""
import copy

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _tiny_llama():
    from transformers import LlamaConfig, LlamaForCausalLM

    torch.manual_seed(0)
    cfg = LlamaConfig(vocab_size=1000, hidden_size=512, intermediate_size=1024,
                      num_hidden_layers=2, num_attention_heads=8, num_key_value_heads=2,
                      max_position_embeddings=512, rms_norm_eps=1e-5)
    cfg._attn_implementation = "sdpa"
    model = LlamaForCausalLM(cfg).to(torch.bfloat16).to(DEV).eval()
    # non-trivial norm weights so the gamma folding is exercised
    for layer in model.model.layers:
        for norm in (layer.input_layernorm, layer.post_attention_layernorm):
            norm.weight.data = (1.0 + 0.1 * torch.randn_like(norm.weight.float())).to(
                norm.weight.dtype)
    return model


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm()).item()


@pytest.mark.parametrize("mode", ["sep", "combined", "swiglu"])
@pytest.mark.parametrize("tokens", [3, 150])
def test_patched_prefill_logits(mode, tokens):
    from src.patch_llama import patch_llama_model

    base = _tiny_llama()
    patched = patch_llama_model(copy.deepcopy(base), variant="V3",
                                combined=(mode == "combined"), swiglu=(mode == "swiglu"))
    ids = torch.randint(0, 1000, (2, tokens), device=DEV, generator=torch.Generator(
        device=DEV).manual_seed(tokens))
    with torch.no_grad():
        ref = base(ids).logits
        out = patched(ids).logits
    assert out.shape == ref.shape
    assert _rel(out, ref) < 3e-2, f"{mode}: relative logit error {_rel(out, ref)}"


def test_gqa_decode_step_matches_sdpa():
    from transformers import DynamicCache

    from src.patch_llama import patch_llama_model

    base = _tiny_llama()
    patched = patch_llama_model(copy.deepcopy(base), variant="V1", swiglu=True, gqa_decode=True)
    assert all(hasattr(l.self_attn, "gqa_decode_module") for l in patched.model.layers)
    ids = torch.randint(0, 1000, (2, 200), device=DEV,
                        generator=torch.Generator(device=DEV).manual_seed(5))
    nxt = torch.randint(0, 1000, (2, 1), device=DEV,
                        generator=torch.Generator(device=DEV).manual_seed(6))
    with torch.no_grad():
        c_ref, c_out = DynamicCache(), DynamicCache()
        base(ids, past_key_values=c_ref, use_cache=True)
        patched(ids, past_key_values=c_out, use_cache=True)
        ref = base(nxt, past_key_values=c_ref, use_cache=True).logits
        out = patched(nxt, past_key_values=c_out, use_cache=True).logits
    assert _rel(out, ref) < 3e-2, f"decode step: relative logit error {_rel(out, ref)}"
