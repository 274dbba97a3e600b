"""Pin the CPU oracle against golden vectors produced by the reference's own
code (tests/golden/make_golden.py)."""
import os

import numpy as np
import pytest
import torch

from oracle import rmsnorm_linear as orc

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "golden_cases.npz")
CASES = ["q_b_small", "kv_b_small", "decode_small", "ragged_bias", "tall_bias"]


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


def _case(g, name):
    M, K, N = (int(v) for v in g[f"{name}__shape"])
    x = orc.from_bf16_bits(g[f"{name}__x"]).reshape(M, K)
    gamma = orc.from_bf16_bits(g[f"{name}__gamma"])
    W = orc.from_bf16_bits(g[f"{name}__W"]).reshape(N, K)
    b = orc.from_bf16_bits(g[f"{name}__b"])
    has_bias = bool(g[f"{name}__has_bias"][0])
    return M, K, N, x, gamma, W, b, has_bias


@pytest.mark.parametrize("name", CASES)
def test_inputs_regenerate_bit_exactly(golden, name):
    """make_inputs is the single source of the seeded inputs."""
    M, K, N, x, gamma, W, *_ = _case(golden, name)
    seed = {"q_b_small": 1234, "kv_b_small": 1235, "decode_small": 1236, "ragged_bias": 1237,
            "tall_bias": 1238}[name]
    x2, g2, W2 = orc.make_inputs(M, K, N, seed=seed)
    assert torch.equal(x.view(torch.int16), x2.view(torch.int16))
    assert torch.equal(gamma.view(torch.int16), g2.view(torch.int16))
    assert torch.equal(W.view(torch.int16), W2.view(torch.int16))


@pytest.mark.parametrize("name", CASES)
def test_fold_gamma_matches_reference_bits(golden, name):
    M, K, N, x, gamma, W, b, _ = _case(golden, name)
    W_new = orc.fold_gamma(W, gamma)
    want = orc.from_bf16_bits(golden[f"{name}__W_new"]).reshape(N, K)
    assert torch.equal(W_new.view(torch.int16), want.view(torch.int16))


def _bf16_ulps_apart(a: torch.Tensor, b: torch.Tensor) -> int:
    """Max distance in bf16 representable steps (sign-magnitude aware)."""
    def key(t):
        i = t.contiguous().view(torch.int16).to(torch.int32)
        return torch.where(i < 0, -(i & 0x7FFF), i)
    return int((key(a) - key(b)).abs().max().item()) if a.numel() else 0


@pytest.mark.parametrize("name", CASES)
def test_unfused_reference_matches(golden, name):
    """linear(SimpleRMSNorm(x)) restated == the reference's output.  CPU bf16
    GEMM blocking may differ between machines, so allow 1 bf16 step."""
    M, K, N, x, gamma, W, b, has_bias = _case(golden, name)
    out = orc.unfused_reference(x, gamma, W, b if has_bias else None, orc.EPS)
    want = orc.from_bf16_bits(golden[f"{name}__ref_out"]).reshape(M, N)
    assert _bf16_ulps_apart(out, want) <= 1


@pytest.mark.parametrize("name", CASES)
def test_torch_rmsnorm_flavour_matches(golden, name):
    M, K, N, x, gamma, W, b, has_bias = _case(golden, name)
    out = orc.unfused_reference(x, gamma, W, b if has_bias else None, orc.EPS, norm="torch")
    want = orc.from_bf16_bits(golden[f"{name}__ref_out_torchnorm"]).reshape(M, N)
    assert _bf16_ulps_apart(out, want) <= 1


@pytest.mark.parametrize("name", CASES)
def test_int8_quantization_matches_reference_bits(golden, name):
    M, K, N, x, gamma, W, b, _ = _case(golden, name)
    W_new = orc.fold_gamma(W, gamma)
    q, scale = orc.quantize_int8_per_output_channel(W_new)
    assert np.array_equal(q.numpy(), golden[f"{name}__q"])
    assert np.array_equal(scale.numpy().view(np.uint32), golden[f"{name}__scale"].view(np.uint32))
    deq = orc.dequantize_int8(q, scale, torch.bfloat16)
    want = orc.from_bf16_bits(golden[f"{name}__deq"]).reshape(N, K)
    assert torch.equal(deq.view(torch.int16), want.view(torch.int16))


@pytest.mark.parametrize("name", CASES)
def test_fused_quantized_matches_reference(golden, name):
    M, K, N, x, gamma, W, b, _ = _case(golden, name)
    q = torch.from_numpy(golden[f"{name}__q"])
    scale = torch.from_numpy(golden[f"{name}__scale"])
    out = orc.fused_quantized(x, q, scale, orc.EPS)
    want = orc.from_bf16_bits(golden[f"{name}__fused_quantized"]).reshape(M, N)
    assert _bf16_ulps_apart(out, want) <= 1


@pytest.mark.parametrize("name", CASES)
def test_truths_agree_with_reference_within_bf16(golden, name):
    """fp32 and fp64 truths vs the reference's bf16 path: the gate the CUDA
    kernel is held to (atol = rtol = 2e-2)."""
    M, K, N, x, gamma, W, b, has_bias = _case(golden, name)
    W_new = orc.fold_gamma(W, gamma)
    bias = b if has_bias else None
    t32 = orc.fp32_truth(x, W_new, bias, orc.EPS)
    t64 = orc.fp64_truth(x.float().numpy(), W_new.float().numpy(),
                         bias.float().numpy() if bias is not None else None, orc.EPS)
    assert np.allclose(t32.numpy(), t64, atol=1e-4, rtol=1e-4)
    ref = orc.from_bf16_bits(golden[f"{name}__ref_out"]).reshape(M, N).float()
    torch.testing.assert_close(t32, ref, atol=2e-2, rtol=2e-2)


def test_combined_folding_matches_reference(golden):
    gamma = orc.from_bf16_bits(golden["combined__gamma"])
    parts = [orc.from_bf16_bits(golden[f"combined__W{i}"]).reshape(-1, 64) for i in range(3)]
    Wc = torch.cat([orc.fold_gamma(p, gamma) for p in parts], dim=0)
    want = orc.from_bf16_bits(golden["combined__W_combined"]).reshape(-1, 64)
    assert torch.equal(Wc.view(torch.int16), want.view(torch.int16))
    assert list(golden["combined__splits"]) == [64, 16, 16]


def test_normalize_reference_is_linear_in_raw():
    """In-place normalize restatement: round(raw*inv_rms + b); with raw the
    exact fp32 GEMM it reproduces the fp32 truth up to one rounding."""
    x, gamma, W = orc.make_inputs(5, 128, 32, seed=3)
    raw = (x.float() @ W.float().t())
    b = torch.zeros(32)
    out = orc.normalize_inplace_reference(x, raw, b, orc.EPS)
    torch.testing.assert_close(out, orc.fp32_truth(x, W, None, orc.EPS), atol=1e-5, rtol=1e-5)
