"""GPU tests of the reference-facing API: denominator_cuda exports, the
FusedRMSNormLinear modules, patch_kimi on a real forward, and the standalone
in-place rmsnorm_normalize kernels."""
import pytest
import torch
import torch.nn as nn

from oracle import rmsnorm_linear as orc
from src import capi, fused_forward, patch_kimi
from src.load_cuda import denominator_cuda

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("config", ["kimi_q_b", "kimi_kv_b"])
@pytest.mark.parametrize("variant", ["V1", "V3"])
def test_reference_kimi_kernel_check(config, variant):
    """The reference's own correctness script (src/test_kimi26_kernels.py:19-52):
    seed 1234, gamma = ones, nn.Linear default init, tokens = 512, bf16,
    max-abs <= 3.5e-2 against linear(norm(x))."""
    M, K, N = orc.CONFIGS[config]
    torch.manual_seed(1234)
    gamma = torch.ones(K, dtype=torch.bfloat16)
    linear = nn.Linear(K, N, bias=False).to(device=DEV, dtype=torch.bfloat16)
    x = torch.randn(M, K, device=DEV, dtype=torch.bfloat16)
    W_new = (linear.weight.detach() * gamma.to(DEV))
    b_new = torch.zeros(N, device=DEV, dtype=torch.bfloat16)
    cls = fused_forward.FusedRMSNormLinearV3 if variant == "V3" else fused_forward.FusedRMSNormLinearV1
    fused = cls(W_new, b_new, K, 1e-5)
    with torch.no_grad():
        actual = fused(x).float().cpu()
    baseline = orc.unfused_reference(x.cpu(), gamma, linear.weight.detach().cpu(), None,
                                     1e-5).float()
    assert (baseline - actual).abs().max().item() <= 3.5e-2


def test_module_leading_dims_and_functional():
    M, K, N = 96, 512, 640
    x, gamma, W = orc.make_inputs(M, K, N, seed=21)
    W_new = orc.fold_gamma(W, gamma)
    b = torch.zeros(N, dtype=torch.bfloat16)
    m = fused_forward.FusedRMSNormLinearV3(W_new.to(DEV), b.to(DEV), K, orc.EPS)
    x3 = x.view(4, 24, K).to(DEV)
    out = m(x3)
    assert out.shape == (4, 24, N)
    out_f = fused_forward.fused_rmsnorm_linear_forward_v1(x3, W_new.to(DEV), b.to(DEV), K, orc.EPS)
    assert torch.equal(out, out_f)
    ref = orc.unfused_reference(x, gamma, W, None, orc.EPS).view(4, 24, N).float()
    torch.testing.assert_close(out.float().cpu(), ref, atol=2e-2, rtol=2e-2)


def test_denominator_cuda_fused_matches_capi():
    M, K, N = 512, 1536, 12288
    x, gamma, W = orc.make_inputs(M, K, N, seed=22)
    W_new = orc.fold_gamma(W, gamma).to(DEV)
    xd = x.to(DEV)
    a = denominator_cuda.fused_rmsnorm_linear(xd, W_new, None, orc.EPS)
    b = capi.fused_rmsnorm_linear(xd, W_new, None, orc.EPS)
    torch.cuda.synchronize()
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))


def test_combined_module_splits():
    M, K = 32, 4096
    x, gamma, W = orc.make_inputs(M, K, 6144, seed=23)
    W_new = orc.fold_gamma(W, gamma)
    b = torch.zeros(6144, dtype=torch.bfloat16)
    m = fused_forward.FusedRMSNormCombinedLinearV1(W_new.to(DEV), b.to(DEV), [4096, 1024, 1024],
                                                   K, orc.EPS)
    q, k, v = m(x.to(DEV))
    assert q.shape == (M, 4096) and k.shape == (M, 1024) and v.shape == (M, 1024)
    assert q.is_contiguous() and k.is_contiguous() and v.is_contiguous()
    ref = orc.unfused_reference(x, gamma, W, None, orc.EPS, norm="torch").float()
    torch.testing.assert_close(torch.cat([q, k, v], -1).float().cpu(), ref, atol=2e-2, rtol=2e-2)


def test_fp32_activations_are_refused_not_rerouted():
    """The fused modules have no fp32 kernel and do not fall back to a library
    GEMM: fp32 input raises a RuntimeError that names the fix."""
    M, K, N = 64, 256, 384
    x, gamma, W = orc.make_inputs(M, K, N, seed=24, dtype=torch.float32)
    W_new = orc.fold_gamma(W, gamma)
    b = torch.zeros(N)
    for cls in (fused_forward.FusedRMSNormLinearV1, fused_forward.FusedRMSNormLinearV3):
        m = cls(W_new.to(DEV), b.to(DEV), K, orc.EPS)
        with pytest.raises(RuntimeError, match="bfloat16 or float16"):
            m(x.to(DEV))
    comb = fused_forward.FusedRMSNormCombinedLinearV1(W_new.to(DEV), b.to(DEV), [256, 128], K,
                                                      orc.EPS)
    with pytest.raises(RuntimeError, match="bfloat16 or float16"):
        comb(x.to(DEV))
    with pytest.raises(RuntimeError, match="bf16 and fp16"):
        denominator_cuda.fused_rmsnorm_linear(x.to(DEV), W_new.to(DEV), b.to(DEV), orc.EPS)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("threads", [256, 512])
@pytest.mark.parametrize("shape", [(7, 100, 50), (64, 1536, 12288), (3, 4096, 6144)])
def test_rmsnorm_normalize_inplace(dtype, threads, shape):
    M, K, N = shape
    x, _, _ = orc.make_inputs(M, K, 8, seed=25, dtype=dtype)
    g = torch.Generator().manual_seed(26)
    raw = torch.randn(M, N, generator=g).to(dtype)
    b = (0.1 * torch.randn(N, generator=g)).to(dtype)
    want = orc.normalize_inplace_reference(x, raw, b, orc.EPS)
    rd = raw.to(DEV)
    fn = denominator_cuda.rmsnorm_normalize_512 if threads == 512 else denominator_cuda.rmsnorm_normalize
    fn(x.to(DEV), rd, b.to(DEV), K, orc.EPS)
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    torch.testing.assert_close(rd.cpu().float(), want.float(), atol=tol, rtol=tol)


def test_rmsnorm_normalize_honours_strides():
    M, K, N = 33, 512, 72
    x, _, _ = orc.make_inputs(M, K, 8, seed=27)
    xbig = torch.full((M, 576), 9.0, dtype=torch.bfloat16)
    xbig[:, :K] = x
    raw = torch.randn(M, N).to(torch.bfloat16)
    rbig = torch.zeros(M, N + 5, dtype=torch.bfloat16)
    rbig[:, :N] = raw
    b = torch.zeros(N, dtype=torch.bfloat16)
    rd = rbig.to(DEV)
    capi.rmsnorm_normalize(xbig.to(DEV)[:, :K], rd[:, :N], b.to(DEV), K, orc.EPS)
    torch.cuda.synchronize()
    want = orc.normalize_inplace_reference(x, raw, b, orc.EPS)
    torch.testing.assert_close(rd[:, :N].cpu().float(), want.float(), atol=1e-2, rtol=1e-2)
    assert torch.all(rd[:, N:].cpu() == 0)


def test_patch_kimi_gpu_forward():
    import sys, os
    sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))
    from make_golden import tiny_deepseek_v3

    model = tiny_deepseek_v3().to(DEV)
    ids = torch.arange(12, device=DEV).view(1, 12)
    with torch.no_grad():
        ref = model(ids).logits.float()
    counts = patch_kimi.patch_kimi_q_lora_norms(model)
    assert counts == {"q_a_layernorm_to_q_b_proj": 3, "kv_a_layernorm_to_kv_b_proj": 3}
    with torch.no_grad():
        got = model(ids).logits.float()
    cos = torch.nn.functional.cosine_similarity(got.flatten(), ref.flatten(), dim=0).item()
    assert cos > 0.999
