"""patch_kimi_q_lora_norms produces the same module tree, counts and folded
weights as the reference's patcher (golden record from the reference run on
the same tiny DeepseekV3), and hands the kernel the strided k_pass view."""
import hashlib
import json
import os
import sys

import pytest
import torch
import torch.nn.functional as F

sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))
from make_golden import tiny_deepseek_v3  # noqa: E402

from src import fused_forward, patch_kimi  # noqa: E402

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "patch_kimi.json")


def _sha(t):
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


@pytest.fixture(scope="module")
def record():
    with open(GOLDEN) as f:
        return json.load(f)


def test_patch_matches_reference(record):
    model = tiny_deepseek_v3()
    counts = patch_kimi.patch_kimi_q_lora_norms(model, device=torch.device("cpu"), variant="V3")
    assert counts == record["counts"]
    again = patch_kimi.patch_kimi_q_lora_norms(model, device=torch.device("cpu"), variant="V3")
    assert again == record["counts_second_call"]
    sd = model.state_dict()
    assert sorted(sd.keys()) == record["state_dict_keys"]
    for k, h in record["fused_sha256"].items():
        assert _sha(sd[k]) == h, k
    types = {n: type(m).__name__ for n, m in model.named_modules()
             if n.endswith(("q_b_proj", "kv_b_proj", "q_a_layernorm", "kv_a_layernorm"))}
    assert types == record["module_types"]


def test_variant_and_layer_resolution_errors():
    model = tiny_deepseek_v3()
    with pytest.raises(ValueError):
        patch_kimi.patch_kimi_q_lora_norms(model, variant="V2")
    with pytest.raises(AttributeError):
        patch_kimi._resolve_text_layers(torch.nn.Linear(2, 2))
    # V1 works too and uses the V1 class
    counts = patch_kimi.patch_kimi_q_lora_norms(model, variant="V1")
    assert counts == {"q_a_layernorm_to_q_b_proj": 3, "kv_a_layernorm_to_kv_b_proj": 3}
    assert isinstance(model.model.layers[0].self_attn.q_b_proj, fused_forward.FusedRMSNormLinearV1)


class _Recorder:
    """Stands in for the CUDA module on CPU: records what reaches the fused
    op and answers with the unfused math."""

    def __init__(self):
        self.calls = []

    def fused_rmsnorm_linear(self, x, W, b, eps):
        self.calls.append((tuple(x.shape), tuple(x.stride()), x.is_contiguous()))
        xf = x.float()
        r = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
        return ((xf @ W.float().t()) * r + b.float()).to(x.dtype)


def test_patched_forward_passes_strided_k_pass(monkeypatch):
    """kv_b_proj receives k_pass = split(compressed_kv)[0], a strided view
    (row stride kv_lora_rank + rope = 40 here); it must reach the op as such."""
    model = tiny_deepseek_v3()
    ref_logits = None
    with torch.no_grad():
        ids = torch.arange(10).view(1, 10)
        ref_logits = model(ids).logits.float()
    rec = _Recorder()
    monkeypatch.setattr(fused_forward, "denominator_cuda", rec)
    patch_kimi.patch_kimi_q_lora_norms(model, device=torch.device("cpu"))
    with torch.no_grad():
        logits = model(ids).logits.float()
    kv_calls = [c for c in rec.calls if c[0][1] == 32]
    q_calls = [c for c in rec.calls if c[0][1] == 48]
    assert len(kv_calls) == 3 and len(q_calls) == 3
    assert all(c[1] == (40, 1) and not c[2] for c in kv_calls)
    assert all(c[2] for c in q_calls)
    # The patched model computes the same function (bf16 model, loose check).
    assert F.cosine_similarity(logits.flatten(), ref_logits.flatten(), dim=0) > 0.999
