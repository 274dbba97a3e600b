"""Generate golden vectors by running the REFERENCE's own Python code on CPU.

Run in a container that has the reference checkout:

    python tests/golden/make_golden.py --reference <path of the reference checkout>

It imports the reference package (``src``) with ``src.load_cuda`` replaced by
a stub -- its CUDA kernels are not needed for any of the functions used here
and nothing gets built -- and records, for small seeded cases:

* the reference's unfused forward ``linear(SimpleRMSNorm(x))`` in bf16
  (src/benchmark_kimi26.py:23-31, :94), and with torch.nn.RMSNorm;
* its gamma folding ``compute_fused_weights_rmsnorm`` (src/weight_transform.py:69-109)
  and ``compute_fused_weights_rmsnorm_combined`` (:142-183);
* its int8 quantizer / dequantizer (src/benchmark_kimi26_quantized.py:30-39) and
  the fused quantized forward composed exactly as its ``fused_quantized``
  closure (:102-106) composes them;
* the module tree produced by ``patch_kimi_q_lora_norms`` on a tiny random
  DeepseekV3 model (src/patch_kimi.py:90-132).

Outputs: tests/golden/golden_cases.npz and tests/golden/patch_kimi.json.
The tests read only those files; the reference is not needed to run them.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys
import types

import numpy as np
import torch
import torch.nn as nn

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from oracle.rmsnorm_linear import bf16_bits, make_inputs  # noqa: E402

# Small cases: name -> (M, K, N, seed, with_bias)
CASES = {
    "q_b_small": (16, 1536, 48, 1234, False),
    "kv_b_small": (16, 512, 64, 1235, False),
    "decode_small": (4, 4096, 16, 1236, False),
    "ragged_bias": (3, 72, 40, 1237, True),
    "tall_bias": (130, 256, 24, 1238, True),
}
EPS = 1e-5


def _load_reference(ref_root: str):
    stub = types.ModuleType("src.load_cuda")
    stub.denominator_cuda = None  # no CUDA build; unused by the functions called here
    sys.modules["src.load_cuda"] = stub
    sys.path.insert(0, ref_root)
    import src  # noqa: F401
    from src import benchmark_kimi26, benchmark_kimi26_quantized, patch_kimi, weight_transform

    return benchmark_kimi26, benchmark_kimi26_quantized, patch_kimi, weight_transform


def _sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def tiny_deepseek_v3(seed: int = 7):
    """A 3-layer random DeepseekV3 model with the q/kv LoRA structure."""
    from transformers import DeepseekV3Config, DeepseekV3ForCausalLM

    cfg = DeepseekV3Config(
        vocab_size=128, hidden_size=64, intermediate_size=96, moe_intermediate_size=32,
        num_hidden_layers=3, num_attention_heads=4, num_key_value_heads=4,
        n_routed_experts=4, n_shared_experts=1, num_experts_per_tok=2, first_k_dense_replace=1,
        n_group=1, topk_group=1, q_lora_rank=48, kv_lora_rank=32, qk_rope_head_dim=8,
        qk_nope_head_dim=16, v_head_dim=16, max_position_embeddings=64,
    )
    torch.manual_seed(seed)
    model = DeepseekV3ForCausalLM(cfg).to(torch.bfloat16)
    # Non-trivial gammas so that folding is visible in the weights.
    g = torch.Generator().manual_seed(seed + 1)
    for layer in model.model.layers:
        for name in ("q_a_layernorm", "kv_a_layernorm"):
            norm = getattr(layer.self_attn, name)
            with torch.no_grad():
                norm.weight.copy_(1.0 + 0.1 * torch.randn(norm.weight.shape, generator=g))
    return model


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True,
                    help="root of the reference checkout (read only)")
    args = ap.parse_args()
    bk, bq, pk, wt = _load_reference(args.reference)

    arrays = {}
    for name, (M, K, N, seed, with_bias) in CASES.items():
        x, gamma, W = make_inputs(M, K, N, seed=seed)
        norm = bk.SimpleRMSNorm(K, eps=EPS).to(torch.bfloat16)
        linear = nn.Linear(K, N, bias=with_bias).to(torch.bfloat16)
        with torch.no_grad():
            norm.weight.copy_(gamma.float())
            linear.weight.copy_(W)
            if with_bias:
                g = torch.Generator().manual_seed(seed + 100)
                linear.bias.copy_((0.5 * torch.randn(N, generator=g)).to(torch.bfloat16))
            ref_out = linear(norm(x))  # reference unfused path, bf16 CPU
            W_new, b_new, h, eps = wt.compute_fused_weights_rmsnorm(norm, linear)
            q, scale = bq.quantize_int8_per_output_channel(W_new)
            deq = bq.dequantize_int8(q, scale, torch.bfloat16)
            # fused_quantized (src/benchmark_kimi26_quantized.py:102-106)
            variance = x.float().pow(2).mean(dim=-1, keepdim=True)
            inv_rms = torch.rsqrt(variance + norm.variance_epsilon).to(torch.bfloat16)
            fq = torch.nn.functional.linear(x * inv_rms, deq)
            # torch.nn.RMSNorm flavour (Llama decode sweep)
            tnorm = nn.RMSNorm(K, eps=EPS).to(torch.bfloat16)
            tnorm.weight.copy_(gamma)
            ref_out_t = linear(tnorm(x))
            W_new_t, _, _, eps_t = wt.compute_fused_weights_rmsnorm(tnorm, linear)
        assert h == K and abs(eps - EPS) < 1e-12 and abs(eps_t - EPS) < 1e-12
        p = f"{name}__"
        arrays[p + "shape"] = np.array([M, K, N], dtype=np.int64)
        arrays[p + "x"] = bf16_bits(x)
        arrays[p + "gamma"] = bf16_bits(gamma)
        arrays[p + "W"] = bf16_bits(W)
        arrays[p + "b"] = bf16_bits(linear.bias.detach() if with_bias else b_new)
        arrays[p + "has_bias"] = np.array([int(with_bias)])
        arrays[p + "ref_out"] = bf16_bits(ref_out)
        arrays[p + "ref_out_torchnorm"] = bf16_bits(ref_out_t)
        arrays[p + "W_new"] = bf16_bits(W_new)
        arrays[p + "W_new_torchnorm"] = bf16_bits(W_new_t)
        arrays[p + "q"] = q.numpy()
        arrays[p + "scale"] = scale.numpy().astype(np.float32)
        arrays[p + "deq"] = bf16_bits(deq)
        arrays[p + "fused_quantized"] = bf16_bits(fq)

    # Combined Q/K/V folding (Llama-3-8B proportions, scaled down 64x).
    g = torch.Generator().manual_seed(99)
    tn = nn.RMSNorm(64, eps=EPS).to(torch.bfloat16)
    with torch.no_grad():
        tn.weight.copy_((1.0 + 0.1 * torch.randn(64, generator=g)).to(torch.bfloat16))
    lins = []
    for n in (64, 16, 16):
        lin = nn.Linear(64, n, bias=False).to(torch.bfloat16)
        with torch.no_grad():
            lin.weight.copy_((torch.randn(n, 64, generator=g) / 8).to(torch.bfloat16))
        lins.append(lin)
    Wc, bc, splits, hc, epsc = wt.compute_fused_weights_rmsnorm_combined(tn, lins)
    arrays["combined__gamma"] = bf16_bits(tn.weight.detach())
    for i, lin in enumerate(lins):
        arrays[f"combined__W{i}"] = bf16_bits(lin.weight.detach())
    arrays["combined__W_combined"] = bf16_bits(Wc)
    arrays["combined__b_combined"] = bf16_bits(bc)
    arrays["combined__splits"] = np.array(splits, dtype=np.int64)

    np.savez_compressed(os.path.join(HERE, "golden_cases.npz"), **arrays)

    # patch_kimi structure on a tiny DeepseekV3.
    model = tiny_deepseek_v3()
    counts = pk.patch_kimi_q_lora_norms(model, device=torch.device("cpu"), variant="V3")
    counts_again = pk.patch_kimi_q_lora_norms(model, device=torch.device("cpu"), variant="V3")
    sd = model.state_dict()
    fused_keys = sorted(k for k in sd if k.endswith(".W_new") or k.endswith(".b_new"))
    record = {
        "counts": counts,
        "counts_second_call": counts_again,
        "state_dict_keys": sorted(sd.keys()),
        "fused_sha256": {k: _sha(sd[k]) for k in fused_keys},
        "module_types": {n: type(m).__name__ for n, m in model.named_modules()
                         if n.endswith(("q_b_proj", "kv_b_proj", "q_a_layernorm",
                                        "kv_a_layernorm"))},
    }
    with open(os.path.join(HERE, "patch_kimi.json"), "w") as f:
        json.dump(record, f, indent=1, sort_keys=True)
    print("wrote", os.path.join(HERE, "golden_cases.npz"), "and patch_kimi.json")
    print("counts", counts, "second call", counts_again)


if __name__ == "__main__":
    main()
