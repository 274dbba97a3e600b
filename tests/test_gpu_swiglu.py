"""GPU parity of the RMSNorm + SwiGLU paths against the CPU oracle.

* frn_fused_rmsnorm_swiglu (one tcgen05 launch: gate and up accumulators of
  the same output columns side by side, silu(g) * u in the epilogue), called
  through the C ABI;
* frn_rmsnorm_swiglu / the module's rmsnorm_swiglu(_512) exports (the
  reference's epilogue over a precomputed [gate | up] GEMM output);
* FusedRMSNormSwiGLUV1/V3 modules.

Gate: torch.allclose(out, reference, atol=2e-2, rtol=2e-2) where reference is
the reference's own FusedRMSNormSwiGLU forward restated on the CPU
(F.linear -> rmsnorm_swiglu); the max-abs error against the fp32 truth is
bounded as well, and the model's unfused silu(gate(norm(x))) * up(norm(x)),
which rounds five times, is held to 3x the tolerance.
"""
import pytest
import torch

from oracle import rmsnorm_linear as orc
from src import capi

pytestmark = pytest.mark.gpu

ATOL = RTOL = 2e-2
DEV = "cuda"


def _inputs(M, K, inter, seed, dtype=torch.bfloat16, bias=False):
    x, gamma, W = orc.make_inputs(M, K, 2 * inter, seed=seed, dtype=dtype)
    Wc = orc.fold_gamma(W, gamma)
    if bias:
        g = torch.Generator().manual_seed(seed + 11)
        b = (0.5 * torch.randn(2 * inter, generator=g)).to(dtype)
    else:
        b = torch.zeros(2 * inter, dtype=dtype)
    return x, gamma, W, Wc, b


def _check_fused(out_gpu, x, gamma, W, Wc, b, inter, tag, has_bias):
    out = out_gpu.float().cpu()
    assert out.shape == (x.shape[0], inter), tag
    assert torch.isfinite(out).all(), tag
    ref = orc.swiglu_module_reference(x, Wc, b, inter, orc.EPS).float()
    torch.testing.assert_close(out, ref, atol=ATOL, rtol=RTOL, msg=lambda m: f"{tag}: {m}")
    if not has_bias:
        # The model's unfused chain rounds to bf16 five times (norm twice, gate,
        # up, silu) before the product, so it sits further from the fp32 truth
        # than either fused path; it is held to a looser bound.
        model = orc.swiglu_unfused_reference(x, gamma, W[:inter], W[inter:], orc.EPS,
                                             norm="simple").float()
        torch.testing.assert_close(out, model, atol=3 * ATOL, rtol=3 * RTOL,
                                   msg=lambda m: f"{tag} vs unfused: {m}")
    truth = orc.swiglu_fp32_truth(x, Wc, b if has_bias else None, inter, orc.EPS)
    err = (out - truth).abs().max().item()
    bound = 2e-2 + 8e-3 * truth.abs().max().item()
    assert err <= bound, f"{tag}: max-abs vs fp32 truth {err} > {bound}"


SHAPES = [
    # (M, K, intermediate)
    (1, 64, 64),
    (7, 512, 192),
    (128, 512, 1024),
    (129, 1536, 224),
    (300, 4096, 512),
    (512, 1536, 1408),
    (1000, 256, 96),
    (256, 64, 4104),
]


@pytest.mark.parametrize("M,K,inter", SHAPES)
def test_fused_swiglu_shapes(M, K, inter):
    x, gamma, W, Wc, b = _inputs(M, K, inter, seed=M + K + inter)
    out = capi.fused_rmsnorm_swiglu(x.to(DEV), Wc.to(DEV), None, orc.EPS)
    torch.cuda.synchronize()
    _check_fused(out, x, gamma, W, Wc, b, inter, f"M={M} K={K} I={inter}", has_bias=False)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_fused_swiglu_bias_and_dtype(dtype):
    M, K, inter = 333, 768, 352
    x, gamma, W, Wc, b = _inputs(M, K, inter, seed=5, dtype=dtype, bias=True)
    out = capi.fused_rmsnorm_swiglu(x.to(DEV), Wc.to(DEV), b.to(DEV), orc.EPS)
    torch.cuda.synchronize()
    _check_fused(out, x, gamma, W, Wc, b, inter, f"bias {dtype}", has_bias=True)


def test_fused_swiglu_strided_rows():
    """x as a row-strided view and out written into a wider buffer."""
    M, K, inter = 200, 512, 256
    x, gamma, W, Wc, b = _inputs(M, K, inter, seed=9)
    xbig = torch.zeros(M, K + 64, dtype=x.dtype)
    xbig[:, 8:8 + K] = x
    xv = xbig.to(DEV)[:, 8:8 + K]
    obig = torch.full((M, inter + 40), 7.0, dtype=x.dtype, device=DEV)
    capi.fused_rmsnorm_swiglu(xv, Wc.to(DEV), None, orc.EPS, out=obig[:, :inter])
    torch.cuda.synchronize()
    _check_fused(obig[:, :inter], x, gamma, W, Wc, b, inter, "strided", has_bias=False)
    assert (obig[:, inter:].float() == 7.0).all(), "wrote past the output columns"


def test_fused_swiglu_llama_mlp_prefill():
    """Llama-3-8B MLP gate/up at 512 prefill tokens (K=4096, I=14336)."""
    M, K, inter = 512, 4096, 14336
    x, gamma, W, Wc, b = _inputs(M, K, inter, seed=77)
    out = capi.fused_rmsnorm_swiglu(x.to(DEV), Wc.to(DEV), None, orc.EPS)
    torch.cuda.synchronize()
    _check_fused(out, x, gamma, W, Wc, b, inter, "llama mlp", has_bias=False)
    assert capi.device_error(0) == 0


@pytest.mark.parametrize("M", [1, 8, 32, 64, 128])
def test_fused_swiglu_decode_path(M):
    """M <= 128 takes the swap-AB split-K decode kernel (64 gate rows over the
    matching 64 up rows per W tile)."""
    K, inter = 4096, 1984
    x, gamma, W, Wc, b = _inputs(M, K, inter, seed=M, bias=(M == 32))
    out = capi.fused_rmsnorm_swiglu(x.to(DEV), Wc.to(DEV), b.to(DEV) if M == 32 else None,
                                    orc.EPS)
    torch.cuda.synchronize()
    _check_fused(out, x, gamma, W, Wc, b, inter, f"decode M={M}", has_bias=(M == 32))


def test_fused_swiglu_llama_mlp_decode():
    """Llama-3-8B MLP gate/up (K=4096, I=14336) at a decode batch of 8."""
    M, K, inter = 8, 4096, 14336
    x, gamma, W, Wc, b = _inputs(M, K, inter, seed=88)
    out = capi.fused_rmsnorm_swiglu(x.to(DEV), Wc.to(DEV), None, orc.EPS)
    torch.cuda.synchronize()
    _check_fused(out, x, gamma, W, Wc, b, inter, "llama mlp decode", has_bias=False)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("threads", [256, 512])
def test_rmsnorm_swiglu_epilogue(dtype, threads):
    M, K, inter = 67, 320, 200
    x, gamma, W, Wc, b = _inputs(M, K, inter, seed=3, dtype=dtype, bias=True)
    raw = torch.nn.functional.linear(x, Wc)
    out = torch.empty(M, inter, dtype=dtype, device=DEV)
    capi.rmsnorm_swiglu(x.to(DEV), raw.to(DEV), out, b.to(DEV), K, inter, orc.EPS, threads)
    torch.cuda.synchronize()
    ref = orc.swiglu_normalize_reference(x, raw, b, inter, orc.EPS).float()
    tol = 1e-5 if dtype == torch.float32 else ATOL
    torch.testing.assert_close(out.float().cpu(), ref, atol=tol, rtol=tol)


def test_module_exports_and_swiglu_modules():
    from src.fused_forward import FusedRMSNormSwiGLUV1, FusedRMSNormSwiGLUV3
    from src.load_cuda import denominator_cuda as dc

    M, K, inter = 96, 1024, 512
    x, gamma, W, Wc, b = _inputs(M, K, inter, seed=21, bias=True)
    ref = orc.swiglu_module_reference(x, Wc, b, inter, orc.EPS).float()
    xd, Wd, bd = x.to(DEV), Wc.to(DEV), b.to(DEV)
    fused = dc.fused_rmsnorm_swiglu(xd, Wd, bd, orc.EPS)
    raw = torch.nn.functional.linear(xd, Wd)
    for fn in (dc.rmsnorm_swiglu, dc.rmsnorm_swiglu_512):
        o = torch.empty(M, inter, dtype=x.dtype, device=DEV)
        fn(xd, raw, o, bd, K, inter, orc.EPS)
        torch.testing.assert_close(o.float().cpu(), ref, atol=ATOL, rtol=RTOL)
    torch.testing.assert_close(fused.float().cpu(), ref, atol=ATOL, rtol=RTOL)
    for cls in (FusedRMSNormSwiGLUV1, FusedRMSNormSwiGLUV3):
        mod = cls(Wd, bd, inter, K, orc.EPS)
        y = mod(xd.view(4, 24, K))
        assert y.shape == (4, 24, inter)
        torch.testing.assert_close(y.reshape(M, inter).float().cpu(), ref, atol=ATOL, rtol=RTOL)
    # fp32 activations are refused (no fp32 tensor-core path, no library fallback)
    mod32 = FusedRMSNormSwiGLUV3(Wd.float(), bd.float(), inter, K, orc.EPS)
    with pytest.raises(RuntimeError, match="bfloat16 or float16"):
        mod32(xd.float())
    with pytest.raises(RuntimeError, match="intermediate columns"):
        dc.rmsnorm_swiglu(xd, raw, torch.empty(M, inter + 8, dtype=x.dtype, device=DEV), bd, K,
                          inter, orc.EPS)
    torch.cuda.synchronize()
    assert capi.device_error(0) == 0
