"""Pins three oracle restatements to the reference's own CUDA kernels, run on
the GPU: the in-place RMSNorm normalize epilogue, the RMSNorm + SwiGLU
epilogue (csrc/denominator_kernel.cu of the reference) and decode-step GQA
attention (csrc/gqa_attention_kernel.cu), built from the reference's sources
by oracle/build_ref.py into oracle/_ref/ (where there is a reference
checkout; the built files travel with the tree).  Each case also checks this
library's kernel for the same op against the reference's output.

Inputs are contiguous with even sizes, as the reference's kernels require
(they index ``x + row * h`` and load two or four elements at a time).
Tolerances: about one rounding of the output type (the reference applies
1/sqrtf under --use_fast_math, the oracle rsqrt), and for GQA the bf16 / fp32
tolerances of the other GQA tests.
"""
import math

import pytest
import torch

from oracle import build_ref
from oracle import gqa_decode as gorc
from oracle import rmsnorm_linear as orc
from src import capi

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = {torch.float32: 2e-5, torch.float16: 2e-3, torch.bfloat16: 1.6e-2}


@pytest.fixture(scope="module")
def ref_den():
    mod = build_ref.load("ref_denominator_cuda")
    if mod is None:
        pytest.skip("oracle/_ref was not built (python oracle/build_ref.py --reference ...)")
    return mod


@pytest.fixture(scope="module")
def ref_gqa():
    mod = build_ref.load("ref_gqa_attention_cuda")
    if mod is None:
        pytest.skip("oracle/_ref was not built (python oracle/build_ref.py --reference ...)")
    return mod


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("v3", [False, True])
@pytest.mark.parametrize("shape", [(64, 512, 1024), (37, 1536, 640), (8, 4096, 6144)])
def test_normalize_oracle_pinned_to_reference_kernel(ref_den, dtype, v3, shape):
    M, K, N = shape
    x, _, _ = orc.make_inputs(M, K, 8, seed=K + N, dtype=dtype)
    g = torch.Generator().manual_seed(M)
    raw = torch.randn(M, N, generator=g).to(dtype)
    b = (0.1 * torch.randn(N, generator=g)).to(dtype)
    ref_out = raw.to(DEV)
    (ref_den.rmsnorm_normalize_512 if v3 else ref_den.rmsnorm_normalize)(
        x.to(DEV), ref_out, b.to(DEV), K, orc.EPS)
    ours = raw.to(DEV)
    capi.rmsnorm_normalize(x.to(DEV), ours, b.to(DEV), K, orc.EPS, 512 if v3 else 256)
    torch.cuda.synchronize()
    ref_out = ref_out.float().cpu()
    tol = TOL[dtype]
    torch.testing.assert_close(orc.normalize_inplace_reference(x, raw, b, orc.EPS).float(),
                               ref_out, atol=tol, rtol=tol)
    torch.testing.assert_close(ours.float().cpu(), ref_out, atol=tol, rtol=tol)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("v3", [False, True])
@pytest.mark.parametrize("shape", [(32, 512, 1024), (9, 4096, 1792)])
def test_swiglu_oracle_pinned_to_reference_kernel(ref_den, dtype, v3, shape):
    M, K, inter = shape
    x, _, _ = orc.make_inputs(M, K, 8, seed=K + inter, dtype=dtype)
    g = torch.Generator().manual_seed(inter)
    raw = (2.0 * torch.randn(M, 2 * inter, generator=g)).to(dtype)
    b = (0.1 * torch.randn(2 * inter, generator=g)).to(dtype)
    ref_out = torch.empty(M, inter, dtype=dtype, device=DEV)
    (ref_den.rmsnorm_swiglu_512 if v3 else ref_den.rmsnorm_swiglu)(
        x.to(DEV), raw.to(DEV), ref_out, b.to(DEV), K, inter, orc.EPS)
    ours = torch.empty(M, inter, dtype=dtype, device=DEV)
    capi.rmsnorm_swiglu(x.to(DEV), raw.to(DEV), ours, b.to(DEV), K, inter, orc.EPS,
                        512 if v3 else 256)
    torch.cuda.synchronize()
    ref_out = ref_out.float().cpu()
    # the reference's expf is __expf under --use_fast_math: a few ulp in fp32
    tol = max(TOL[dtype], 1e-4)
    torch.testing.assert_close(orc.swiglu_normalize_reference(x, raw, b, inter, orc.EPS).float(),
                               ref_out, atol=tol, rtol=tol)
    torch.testing.assert_close(ours.float().cpu(), ref_out, atol=tol, rtol=tol)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("shape", [(2, 32, 8, 128, 300), (3, 16, 4, 64, 77), (1, 8, 1, 128, 64)])
def test_gqa_oracle_pinned_to_reference_kernel(ref_gqa, dtype, shape):
    B, Hq, Hkv, D, T = shape
    q, k, v = gorc.make_gqa_inputs(B, Hq, Hkv, D, T, seed=T, dtype=dtype)
    scale = 1.0 / math.sqrt(D)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    out_v3 = torch.empty_like(qd)
    ref_gqa.gqa_decode_v3(qd, kd, vd, out_v3, Hq // Hkv, scale)
    out_v2 = torch.empty_like(qd)
    ref_gqa.gqa_decode_v2(qd, kd, vd, out_v2, scale)
    ours = capi.gqa_decode_attention(qd, kd, vd, scale)
    torch.cuda.synchronize()
    tol = 1e-4 if dtype == torch.float32 else 2e-2
    want = gorc.gqa_decode_reference(q, k, v, scale)
    for ref_out in (out_v3, out_v2):
        torch.testing.assert_close(want, ref_out.float().cpu(), atol=tol, rtol=tol)
        torch.testing.assert_close(ours.float().cpu(), ref_out.float().cpu(), atol=tol, rtol=tol)
