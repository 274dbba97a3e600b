"""GPU parity of the fused RMSNorm -> Linear kernel, called through the C ABI
(ctypes on libfrn_b200.so), against the CPU oracle on the same seeded inputs.

Gate (bf16 / fp16): torch.allclose(out, reference_unfused, atol=2e-2,
rtol=2e-2) where reference_unfused is the reference's own
linear(SimpleRMSNorm(x)) restated on the CPU; the max-abs error against the
fp32 truth is reported and bounded as well.
"""
import pytest
import torch

from oracle import rmsnorm_linear as orc
from src import capi

pytestmark = pytest.mark.gpu

ATOL = RTOL = 2e-2
DEV = "cuda"


def _inputs(M, K, N, seed, dtype=torch.bfloat16, bias=False):
    x, gamma, W = orc.make_inputs(M, K, N, seed=seed, dtype=dtype)
    W_new = orc.fold_gamma(W, gamma)
    b = None
    if bias:
        g = torch.Generator().manual_seed(seed + 7)
        b = (0.5 * torch.randn(N, generator=g)).to(dtype)
    return x, gamma, W, W_new, b


def _check(out_gpu, x, gamma, W, W_new, b, tag=""):
    out = out_gpu.float().cpu()
    ref = orc.unfused_reference(x, gamma, W, b, orc.EPS).float()
    truth = orc.fp32_truth(x, W_new, b, orc.EPS)
    assert torch.isfinite(out).all(), tag
    torch.testing.assert_close(out, ref, atol=ATOL, rtol=RTOL, msg=lambda m: f"{tag}: {m}")
    err = (out - truth).abs().max().item()
    # one output rounding plus fp32 accumulation-order noise
    bound = 2e-2 + 8e-3 * truth.abs().max().item()
    assert err <= bound, f"{tag}: max-abs vs fp32 truth {err} > {bound}"
    return err


@pytest.mark.parametrize("config", ["kimi_q_b", "kimi_kv_b", "kimi_q_b_long", "kimi_kv_b_long",
                                    "decode_m1", "decode_m8", "decode_m32", "decode_m128"])
def test_baseline_configs_full_size(config):
    M, K, N = orc.CONFIGS[config]
    x, gamma, W, W_new, b = _inputs(M, K, N, seed=1234)
    out = capi.fused_rmsnorm_linear(x.to(DEV), W_new.to(DEV), None, orc.EPS)
    torch.cuda.synchronize()
    _check(out, x, gamma, W, W_new, b, config)


ALL_KERNELS = [capi.FRN_KERNEL_TILE_N128, capi.FRN_KERNEL_TILE_N192, capi.FRN_KERNEL_TILE_N256,
               capi.FRN_KERNEL_PAIR_N128, capi.FRN_KERNEL_PAIR_N160, capi.FRN_KERNEL_PAIR_N192,
               capi.FRN_KERNEL_PAIR_N224, capi.FRN_KERNEL_PAIR_N256, capi.FRN_KERNEL_WIDE_N128,
               capi.FRN_KERNEL_WIDE_N192, capi.FRN_KERNEL_WIDE_N224, capi.FRN_KERNEL_WIDE_N256,
               capi.FRN_KERNEL_WIDE_N176]


@pytest.mark.parametrize("kernel", ALL_KERNELS)
@pytest.mark.parametrize("shape", [(512, 1536, 12288), (512, 512, 16384), (300, 1536, 1000),
                                   (129, 72, 264)])
def test_every_tile_width(kernel, shape):
    M, K, N = shape
    x, gamma, W, W_new, b = _inputs(M, K, N, seed=11, bias=True)
    out = capi.fused_rmsnorm_linear(x.to(DEV), W_new.to(DEV), b.to(DEV), orc.EPS, kernel=kernel)
    torch.cuda.synchronize()
    _check(out, x, gamma, W, W_new, b, f"kernel{kernel} {shape}")


@pytest.mark.parametrize("M", [1, 2, 3, 127, 128, 129, 255, 257])
@pytest.mark.parametrize("K,N", [(8, 8), (72, 40), (520, 200), (1536, 264)])
def test_ragged_shapes_with_bias(M, K, N):
    x, gamma, W, W_new, b = _inputs(M, K, N, seed=M * 31 + K + N, bias=True)
    out = capi.fused_rmsnorm_linear(x.to(DEV), W_new.to(DEV), b.to(DEV), orc.EPS)
    torch.cuda.synchronize()
    _check(out, x, gamma, W, W_new, b, f"M{M} K{K} N{N}")


def test_strided_x_rows_like_deepseek_k_pass():
    """kv_b's input is split(compressed_kv, [512, 64])[0]: row stride 576."""
    M, K, N = 512, 512, 16384
    x, gamma, W, W_new, b = _inputs(M, K, N, seed=5)
    full = torch.zeros(M, 576, dtype=torch.bfloat16)
    full[:, :K] = x
    full[:, K:] = 7.0  # garbage that must not enter the RMS
    xs = full.to(DEV)[:, :K]
    assert xs.stride() == (576, 1)
    out = capi.fused_rmsnorm_linear(xs, W_new.to(DEV), None, orc.EPS)
    torch.cuda.synchronize()
    _check(out, x, gamma, W, W_new, b, "strided")


def test_output_row_stride_and_untouched_padding():
    M, K, N = 200, 256, 136
    x, gamma, W, W_new, b = _inputs(M, K, N, seed=6, bias=True)
    buf = torch.full((M, N + 24), 3.0, dtype=torch.bfloat16, device=DEV)
    out = buf[:, :N]
    capi.fused_rmsnorm_linear(x.to(DEV), W_new.to(DEV), b.to(DEV), orc.EPS, out=out)
    torch.cuda.synchronize()
    _check(out, x, gamma, W, W_new, b, "out stride")
    assert torch.all(buf[:, N:] == 3.0), "kernel wrote outside the output view"


def test_fp16():
    M, K, N = 256, 1536, 2048
    x, gamma, W, W_new, b = _inputs(M, K, N, seed=8, dtype=torch.float16, bias=True)
    out = capi.fused_rmsnorm_linear(x.to(DEV), W_new.to(DEV), b.to(DEV), orc.EPS)
    torch.cuda.synchronize()
    assert out.dtype == torch.float16
    _check(out, x, gamma, W, W_new, b, "fp16")


@pytest.mark.parametrize("kernel", ALL_KERNELS)
def test_strided_fp16_bias_every_kernel(kernel):
    M, K, N = 384, 576, 1040
    x, gamma, W, W_new, b = _inputs(M, K, N, seed=12, dtype=torch.float16, bias=True)
    full = torch.zeros(M, K + 64, dtype=torch.float16)
    full[:, :K] = x
    out = capi.fused_rmsnorm_linear(full.to(DEV)[:, :K], W_new.to(DEV), b.to(DEV), orc.EPS,
                                    kernel=kernel)
    torch.cuda.synchronize()
    _check(out, x, gamma, W, W_new, b, f"kernel{kernel} strided fp16")


@pytest.mark.parametrize("M", [1, 2, 7, 8, 16, 17, 32, 33, 64, 100, 128])
@pytest.mark.parametrize("K,N", [(4096, 6144), (512, 16384), (72, 136), (1536, 1000)])
def test_decode_kernel(M, K, N):
    """Swap-AB split-K cluster kernel for M <= 128 (the Llama-3-8B QKV decode
    sweep is K=4096, N=6144), against the oracle; bias on odd M."""
    x, gamma, W, W_new, b = _inputs(M, K, N, seed=M + 3 * K + N, bias=(M % 2 == 1))
    bd = b.to(DEV) if b is not None else None
    out = capi.fused_rmsnorm_linear(x.to(DEV), W_new.to(DEV), bd, orc.EPS,
                                    kernel=capi.FRN_KERNEL_DECODE)
    torch.cuda.synchronize()
    _check(out, x, gamma, W, W_new, b, f"decode M{M} K{K} N{N}")


@pytest.mark.parametrize("M", [1, 9, 64, 128])
@pytest.mark.parametrize("K,N", [(2048, 1024), (1280, 3200), (1792, 2432)])
def test_decode_kernel_cluster_sizes(M, K, N):
    """Shapes that ask for k-splits of 8, 5 and 7 CTAs per cluster (the
    one-wave cap may lower the last two): other owner / slot mappings of the
    cluster reduction than the Llama-3-8B shape's 2, with the receive buffer
    in its own space (M <= 64) and over the W stages (M = 128)."""
    x, gamma, W, W_new, b = _inputs(M, K, N, seed=7 * M + K + N, bias=True)
    out = capi.fused_rmsnorm_linear(x.to(DEV), W_new.to(DEV), b.to(DEV), orc.EPS,
                                    kernel=capi.FRN_KERNEL_DECODE)
    torch.cuda.synchronize()
    _check(out, x, gamma, W, W_new, b, f"decode M{M} K{K} N{N}")


def test_decode_strided_fp16_and_determinism():
    M, K, N = 24, 4096, 6144
    x, gamma, W, W_new, b = _inputs(M, K, N, seed=31, dtype=torch.float16, bias=True)
    full = torch.zeros(M, K + 64, dtype=torch.float16)
    full[:, :K] = x
    xs, wd, bd = full.to(DEV)[:, :K], W_new.to(DEV), b.to(DEV)
    o1 = capi.fused_rmsnorm_linear(xs, wd, bd, orc.EPS, kernel=capi.FRN_KERNEL_DECODE)
    o2 = capi.fused_rmsnorm_linear(xs, wd, bd, orc.EPS, kernel=capi.FRN_KERNEL_DECODE)
    torch.cuda.synchronize()
    assert torch.equal(o1.view(torch.int16), o2.view(torch.int16))
    _check(o1, x, gamma, W, W_new, b, "decode strided fp16")


def test_decode_rejects_large_m():
    x = torch.zeros(129, 64, dtype=torch.bfloat16, device=DEV)
    w = torch.zeros(64, 64, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(capi.FrnError):
        capi.fused_rmsnorm_linear(x, w, None, orc.EPS, kernel=capi.FRN_KERNEL_DECODE)


def test_deterministic_bits():
    M, K, N = 512, 1536, 12288
    x, gamma, W, W_new, b = _inputs(M, K, N, seed=9)
    xd, wd = x.to(DEV), W_new.to(DEV)
    o1 = capi.fused_rmsnorm_linear(xd, wd, None, orc.EPS)
    o2 = capi.fused_rmsnorm_linear(xd, wd, None, orc.EPS)
    torch.cuda.synchronize()
    assert torch.equal(o1.view(torch.int16), o2.view(torch.int16))


def test_zero_rows_and_large_values():
    """An all-zero row gives bias only (inv_rms = rsqrt(eps) times a zero
    dot product); rows of large magnitude normalise without overflow."""
    M, K, N = 130, 512, 256
    x, gamma, W, W_new, b = _inputs(M, K, N, seed=10, bias=True)
    x[3] = 0
    x[100] = x[100] * 3000.0
    out = capi.fused_rmsnorm_linear(x.to(DEV), W_new.to(DEV), b.to(DEV), orc.EPS)
    torch.cuda.synchronize()
    _check(out, x, gamma, W, W_new, b, "zero/large rows")
    torch.testing.assert_close(out[3].float().cpu(), b.float(), atol=0, rtol=0)


def test_device_error_word_clear():
    torch.cuda.synchronize()
    assert capi.device_error(torch.cuda.current_device()) == 0
