"""GPU parity of the split-output fused RMSNorm -> Linear (combined Q/K/V):
one launch whose output columns land directly in separate tensors, checked
part by part against the CPU oracle's full [M, N] result (the reference's
FusedRMSNormCombinedLinear forward is F.linear + normalize, then split +
.contiguous(); src/fused_forward.py:194-251)."""
import pytest
import torch

from oracle import rmsnorm_linear as orc
from src import capi

pytestmark = pytest.mark.gpu

ATOL = RTOL = 2e-2
DEV = "cuda"
LLAMA_QKV = [4096, 1024, 1024]


def _inputs(M, K, N, seed, bias=False, dtype=torch.bfloat16):
    x, gamma, W = orc.make_inputs(M, K, N, seed=seed, dtype=dtype)
    Wn = orc.fold_gamma(W, gamma)
    b = None
    if bias:
        g = torch.Generator().manual_seed(seed + 3)
        b = (0.5 * torch.randn(N, generator=g)).to(dtype)
    return x, gamma, W, Wn, b


def _check_parts(parts, x, gamma, W, Wn, b, sizes, tag):
    ref = orc.unfused_reference(x, gamma, W, b, orc.EPS, norm="torch").float()
    truth = orc.fp32_truth(x, Wn, b, orc.EPS)
    c0 = 0
    for i, (p, c) in enumerate(zip(parts, sizes)):
        assert p.shape == (x.shape[0], c), f"{tag} part {i}"
        got = p.float().cpu()
        torch.testing.assert_close(got, ref[:, c0:c0 + c], atol=ATOL, rtol=RTOL,
                                   msg=lambda m: f"{tag} part {i}: {m}")
        err = (got - truth[:, c0:c0 + c]).abs().max().item()
        assert err <= 2e-2 + 8e-3 * truth.abs().max().item(), f"{tag} part {i}: {err}"
        c0 += c


@pytest.mark.parametrize("M", [1, 8, 32, 128, 129, 512])
def test_llama_qkv_split(M):
    K, N = 4096, sum(LLAMA_QKV)
    x, gamma, W, Wn, b = _inputs(M, K, N, seed=40 + M)
    parts = capi.fused_rmsnorm_linear_split(x.to(DEV), Wn.to(DEV), None, orc.EPS, LLAMA_QKV)
    torch.cuda.synchronize()
    assert all(p.is_contiguous() for p in parts)
    _check_parts(parts, x, gamma, W, Wn, b, LLAMA_QKV, f"qkv M={M}")


@pytest.mark.parametrize("sizes", [[64, 136, 8], [512, 256, 256, 1024], [2048]])
def test_ragged_parts_decode(sizes):
    """Decode token counts accept any 8-column multiples, 1 to 4 parts."""
    M, K = 24, 1024
    N = sum(sizes)
    x, gamma, W, Wn, b = _inputs(M, K, N, seed=sum(sizes), bias=True)
    parts = capi.fused_rmsnorm_linear_split(x.to(DEV), Wn.to(DEV), b.to(DEV), orc.EPS, sizes)
    torch.cuda.synchronize()
    _check_parts(parts, x, gamma, W, Wn, b, sizes, f"ragged {sizes}")


def test_strided_part_buffers_and_guards():
    """Parts written into wider row-strided buffers; columns past each part
    stay untouched."""
    M, K = 300, 512
    sizes = [256, 128, 640]
    N = sum(sizes)
    x, gamma, W, Wn, b = _inputs(M, K, N, seed=8)
    bufs = [torch.full((M, c + 64), 3.0, dtype=torch.bfloat16, device=DEV) for c in sizes]
    views = [buf[:, :c] for buf, c in zip(bufs, sizes)]
    capi.fused_rmsnorm_linear_split(x.to(DEV), Wn.to(DEV), None, orc.EPS, sizes, outs=views)
    torch.cuda.synchronize()
    _check_parts(views, x, gamma, W, Wn, b, sizes, "strided")
    for buf, c in zip(bufs, sizes):
        assert (buf[:, c:].float() == 3.0).all()


def test_split_rejections():
    x, gamma, W, Wn, b = _inputs(256, 128, 192, seed=1)
    xd, wd = x.to(DEV), Wn.to(DEV)
    with pytest.raises(capi.FrnError, match="multiples of 64"):
        capi.fused_rmsnorm_linear_split(xd, wd, None, orc.EPS, [96, 96])
    with pytest.raises(capi.FrnError, match="sum to"):
        capi.fused_rmsnorm_linear_split(xd, wd, None, orc.EPS, [64, 64])
    with pytest.raises(capi.FrnError, match="multiple of 8"):
        capi.fused_rmsnorm_linear_split(xd[:8], wd, None, orc.EPS, [100, 92])


@pytest.mark.parametrize("M", [4, 512])
def test_combined_modules_return_contiguous_parts(M):
    from src.fused_forward import FusedRMSNormCombinedLinearV1, FusedRMSNormCombinedLinearV3

    K = 1024
    sizes = [1024, 256, 256]
    N = sum(sizes)
    x, gamma, W, Wn, b = _inputs(M, K, N, seed=M, bias=True)
    for cls in (FusedRMSNormCombinedLinearV1, FusedRMSNormCombinedLinearV3):
        mod = cls(Wn.to(DEV), b.to(DEV), sizes, K, orc.EPS)
        parts = mod(x.to(DEV).view(1, M, K))
        assert [tuple(p.shape) for p in parts] == [(1, M, c) for c in sizes]
        assert all(p.is_contiguous() for p in parts)
        _check_parts([p.view(M, -1) for p in parts], x, gamma, W, Wn, b, sizes, cls.__name__)
    assert capi.device_error(0) == 0
