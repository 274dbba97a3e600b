"""GPU parity of the int8-weight path: the quantizer against the reference's
quantize_int8_per_output_channel (bit-exact), and the fused int8 kernel
against the reference's dequantized forward (fused_quantized) within
atol = rtol = 2e-2, and against the exact int8 math in fp32."""
import pytest
import torch

from oracle import rmsnorm_linear as orc
from src import capi

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("shape", [(12288, 1536), (16384, 512), (40, 72), (6144, 4096)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_quantizer_bit_exact(shape, dtype):
    N, K = shape
    _, gamma, W = orc.make_inputs(1, K, N, seed=N + K, dtype=dtype)
    W_new = orc.fold_gamma(W, gamma)
    q_ref, s_ref = orc.quantize_int8_per_output_channel(W_new)
    q, s = capi.quantize_int8_per_channel(W_new.to(DEV))
    torch.cuda.synchronize()
    assert torch.equal(q.cpu(), q_ref)
    assert torch.equal(s.cpu().view(torch.int32), s_ref.float().view(torch.int32))


def _case(M, K, N, seed, bias=False, dtype=torch.bfloat16):
    x, gamma, W = orc.make_inputs(M, K, N, seed=seed, dtype=dtype)
    W_new = orc.fold_gamma(W, gamma)
    q, s = orc.quantize_int8_per_output_channel(W_new)
    b = None
    if bias:
        g = torch.Generator().manual_seed(seed + 9)
        b = (0.5 * torch.randn(N, generator=g)).to(dtype)
    return x, q, s, b


def _check(out, x, q, s, b, tag):
    out = out.float().cpu()
    ref = orc.fused_quantized(x, q, s, orc.EPS, dtype=x.dtype).float()
    if b is not None:
        ref = ref + b.float()
    truth = orc.int8_fp32_truth(x, q, s, b, orc.EPS)
    assert torch.isfinite(out).all(), tag
    torch.testing.assert_close(out, ref, atol=2e-2, rtol=2e-2, msg=lambda m: f"{tag}: {m}")
    torch.testing.assert_close(out, truth, atol=1e-2, rtol=1e-2, msg=lambda m: f"{tag}: {m}")


@pytest.mark.parametrize("shape", [(2048, 1536, 12288), (512, 1536, 12288), (512, 512, 16384),
                                   (4096, 512, 16384), (300, 1536, 1000), (129, 64, 264),
                                   (1, 256, 128)])
def test_fused_int8(shape):
    M, K, N = shape
    x, q, s, b = _case(M, K, N, seed=M + K + N, bias=(M % 2 == 1))
    out = capi.fused_rmsnorm_linear_w8(x.to(DEV), q.to(DEV), s.to(DEV),
                                       b.to(DEV) if b is not None else None, orc.EPS)
    torch.cuda.synchronize()
    _check(out, x, q, s, b, f"int8 {shape}")


def test_fused_int8_fp16_strided():
    M, K, N = 384, 512, 1024
    x, q, s, b = _case(M, K, N, seed=77, bias=True, dtype=torch.float16)
    full = torch.zeros(M, 576, dtype=torch.float16)
    full[:, :K] = x
    out = capi.fused_rmsnorm_linear_w8(full.to(DEV)[:, :K], q.to(DEV), s.to(DEV), b.to(DEV),
                                       orc.EPS)
    torch.cuda.synchronize()
    _check(out, x, q, s, b, "int8 fp16 strided")


def test_int8_module_and_patch_variant():
    from src.quantized import FusedRMSNormLinearInt8

    M, K, N = 256, 1536, 2048
    x, gamma, W = orc.make_inputs(M, K, N, seed=5)
    W_new = orc.fold_gamma(W, gamma)
    mod = FusedRMSNormLinearInt8(W_new.to(DEV), torch.zeros(N, dtype=torch.bfloat16, device=DEV),
                                 K, orc.EPS)
    assert set(mod.state_dict()) == {"qweight", "w_scale", "b_new"}
    out = mod(x.view(4, 64, K).to(DEV)).view(M, N)
    q, s = orc.quantize_int8_per_output_channel(W_new)
    _check(out, x, q, s, None, "int8 module")


def test_int8_rejects_bad_alignment():
    x = torch.zeros(4, 72, dtype=torch.bfloat16, device=DEV)
    q = torch.zeros(8, 72, dtype=torch.int8, device=DEV)
    s = torch.ones(8, device=DEV)
    with pytest.raises(capi.FrnError):
        capi.fused_rmsnorm_linear_w8(x, q, s, None, 1e-5)


@pytest.mark.parametrize("pair", [
    ((256, 1536, 12288), (256, 512, 16384)),   # one 8-GPU shard of the int8 stack's layer
    ((200, 1536, 1000), (129, 64, 264)),        # ragged, different M, N and K, one launch
    ((256, 512, 16384), (1, 256, 128)),
    ((1024, 1536, 12288), (1024, 512, 16384)),  # more than one m-block: two launches
    ((300, 1536, 1000), (129, 64, 264)),
])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_grouped_int8_matches_separate_calls(pair, dtype):
    """Two independent problems through the grouped entry point (one launch
    while both have <= 256 rows): each output against the oracle and
    bit-identical to its own single-problem launch (same per-element k-order
    and epilogue, whatever the tile width)."""
    probs, cases = [], []
    for i, (M, K, N) in enumerate(pair):
        x, q, s, b = _case(M, K, N, seed=M + K + N + i, bias=(i == 1), dtype=dtype)
        cases.append((x, q, s, b))
        out = torch.empty(M, N, dtype=dtype, device=DEV)
        probs.append((x.to(DEV), q.to(DEV), s.to(DEV), b.to(DEV) if b is not None else None, out))
    outs = capi.fused_rmsnorm_linear_w8_grouped(probs, orc.EPS)
    singles = [capi.fused_rmsnorm_linear_w8(p[0], p[1], p[2], p[3], orc.EPS) for p in probs]
    torch.cuda.synchronize()
    for (x, q, s, b), o, o1, shape in zip(cases, outs, singles, pair):
        _check(o, x, q, s, b, f"grouped {shape}")
        assert torch.equal(o.view(torch.int16), o1.view(torch.int16)), f"grouped {shape}"


def test_grouped_int8_edge_cases():
    """One problem with no rows runs the other alone; more than two problems
    and mixed x dtypes are rejected."""
    x, q, s, b = _case(256, 512, 16384, seed=5)
    xd, qd, sd = x.to(DEV), q.to(DEV), s.to(DEV)
    out = torch.empty(256, 16384, dtype=torch.bfloat16, device=DEV)
    empty = torch.empty(0, 512, dtype=torch.bfloat16, device=DEV)
    eout = torch.empty(0, 16384, dtype=torch.bfloat16, device=DEV)
    capi.fused_rmsnorm_linear_w8_grouped([(empty, qd, sd, None, eout), (xd, qd, sd, None, out)],
                                         orc.EPS)
    torch.cuda.synchronize()
    _check(out, x, q, s, None, "grouped with an empty problem")
    arr = (capi.W8Linear * 3)()
    rc = capi.lib().frn_fused_rmsnorm_linear_w8_grouped(capi.FRN_DTYPE_BF16, arr, 3, 1e-6, None)
    assert rc == capi.FRN_ERR_INVALID_ARGUMENT


def test_int8_stack_groups_layer_pairs():
    """fused_stack_token_parallel with int8 layers: consecutive layers share a
    launch; every output equals its own single-layer call."""
    from src import multigpu
    from src.load_cuda import denominator_cuda

    shapes = [(200, 1536, 12288), (200, 512, 16384), (200, 1536, 12288)]  # odd count: last alone
    xs, layers = [], []
    for i, (M, K, N) in enumerate(shapes):
        x, q, s, _ = _case(M, K, N, seed=40 + i)
        xs.append(x.to(DEV))
        layers.append(((q.to(DEV), s.to(DEV)), None))
    outs = multigpu.fused_stack_token_parallel(xs, layers, orc.EPS)
    for x, ((q, s), _), o in zip(xs, layers, outs):
        ref = denominator_cuda.fused_rmsnorm_linear_w8(x, q, s, None, orc.EPS)
        torch.cuda.synchronize()
        assert torch.equal(o.view(torch.int16), ref.view(torch.int16))
