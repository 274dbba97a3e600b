"""denominator_cuda / fused_forward surface on CPU: names, buffers, errors."""
import pytest
import torch

from src import fused_forward
from src.load_cuda import denominator_cuda

REFERENCE_EXPORTS = [
    "compute_denominator", "denominator_normalize", "compute_denominator_welford",
    "denominator_normalize_welford_512", "rmsnorm_normalize", "rmsnorm_normalize_512",
    "rmsnorm_swiglu", "rmsnorm_swiglu_512",
]


def test_module_exports():
    for name in REFERENCE_EXPORTS + ["fused_rmsnorm_linear", "device_error"]:
        if name.startswith("rmsnorm_swiglu"):
            continue  # added with the fused SwiGLU epilogue
        assert hasattr(denominator_cuda, name), name


def test_loaded_from_tree():
    import os

    here = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    assert os.path.realpath(denominator_cuda.__file__).startswith(os.path.realpath(here))


def test_cpu_tensors_rejected_like_reference():
    x = torch.randn(4, 8, dtype=torch.bfloat16)
    raw = torch.randn(4, 16, dtype=torch.bfloat16)
    b = torch.zeros(16, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="All tensors must be on CUDA"):
        denominator_cuda.rmsnorm_normalize(x, raw, b, 8, 1e-5)
    with pytest.raises(RuntimeError, match="All tensors must be on CUDA"):
        denominator_cuda.rmsnorm_normalize_512(x, raw, b, 8, 1e-5)
    with pytest.raises(RuntimeError, match="All tensors must be on CUDA"):
        denominator_cuda.fused_rmsnorm_linear(x, torch.randn(16, 8, dtype=torch.bfloat16), b, 1e-5)
    with pytest.raises(RuntimeError, match="x must be 2D"):
        denominator_cuda.rmsnorm_normalize(x.view(-1), raw, b, 8, 1e-5)


def test_layernorm_exports_say_out_of_scope():
    with pytest.raises(RuntimeError, match="LayerNorm"):
        denominator_cuda.compute_denominator(torch.randn(2, 2))


@pytest.mark.parametrize("cls", [fused_forward.FusedRMSNormLinearV1,
                                 fused_forward.FusedRMSNormLinearV3])
def test_module_buffers_and_state_dict(cls):
    W = torch.randn(16, 8, dtype=torch.bfloat16)
    b = torch.zeros(16, dtype=torch.bfloat16)
    m = cls(W, b, 8, 1e-5)
    assert set(m.state_dict()) == {"W_new", "b_new"}
    assert m.h == 8 and m.eps == 1e-5
    with pytest.raises(RuntimeError, match="All tensors must be on CUDA"):
        m(torch.randn(2, 3, 8, dtype=torch.bfloat16))


def test_combined_and_swiglu_buffers():
    W = torch.randn(24, 8, dtype=torch.bfloat16)
    b = torch.zeros(24, dtype=torch.bfloat16)
    c = fused_forward.FusedRMSNormCombinedLinearV3(W, b, [16, 4, 4], 8, 1e-5)
    assert set(c.state_dict()) == {"W_combined", "b_combined"}
    s = fused_forward.FusedRMSNormSwiGLUV1(W, b, 12, 8, 1e-5)
    assert set(s.state_dict()) == {"W_combined", "b_combined"} and s.intermediate == 12


def test_patch_llama_structure_on_cpu():
    """patch_llama attaches the reference's module names and replaces the
    forwards; building the fused modules needs no GPU."""
    import pytest as _pytest
    from transformers import LlamaConfig, LlamaForCausalLM

    from src.patch_llama import patch_llama_model

    cfg = LlamaConfig(vocab_size=64, hidden_size=128, intermediate_size=256,
                      num_hidden_layers=2, num_attention_heads=2, num_key_value_heads=1)
    for kw, attrs in (({}, ("fused_q_proj", "fused_gate_proj")),
                      ({"combined": True}, ("fused_qkv", "fused_gate_up")),
                      ({"swiglu": True, "gqa_decode": True},
                       ("fused_qkv", "fused_gate_up_swiglu", "gqa_decode_module"))):
        model = patch_llama_model(LlamaForCausalLM(cfg), device="cpu", **kw)
        for layer in model.model.layers:
            owners = (layer.self_attn, layer.mlp)
            for a in attrs:
                assert any(hasattr(o, a) for o in owners), (kw, a)
            assert "forward" in vars(layer) and "forward" in vars(layer.self_attn)
    with _pytest.raises(ValueError, match="Unknown variant"):
        patch_llama_model(LlamaForCausalLM(cfg), device="cpu", variant="V2")


def test_fp32_activations_refused_before_any_launch():
    """fp32 has no tensor-core path here and no library-GEMM fallback: the
    modules raise before touching the device."""
    W = torch.randn(16, 8)
    b = torch.zeros(16)
    for cls in (fused_forward.FusedRMSNormLinearV1, fused_forward.FusedRMSNormLinearV3):
        with pytest.raises(RuntimeError, match="bfloat16 or float16"):
            cls(W, b, 8, 1e-5)(torch.randn(2, 8))
    sw = fused_forward.FusedRMSNormSwiGLUV1(torch.randn(16, 8), torch.zeros(16), 8, 8, 1e-5)
    with pytest.raises(RuntimeError, match="bfloat16 or float16"):
        sw(torch.randn(2, 8))
