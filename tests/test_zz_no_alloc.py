"""The allocation-free GQA decode entry point (frn_gqa_decode_attention_noalloc),
called through the C ABI.

It exists for hosts that cannot call cudaMalloc while decoding (all device
memory reserved up front by their own pool, or allocation banned on the decode
path).  Only fp32 calls use its static scratch array: they run the CUDA-core
kernel, whose context split parks partial results there for a merge launch.
bf16 / fp16 calls run the tensor-core kernel, which merges on chip.

Each case makes two calls in a row with different inputs (the second finds
the first one's partials in the shared array) and checks both against the
allocating entry point (frn_gqa_decode_attention with its workspace) and the
fp64 oracle, within the GQA tolerances of the other GPU tests.  The file is
collected last, so a run that stops at the first failure has already run every
other test; it passes alone in a fresh process as well.
"""
import math

import pytest
import torch

from oracle import gqa_decode as orc
from src import capi

pytestmark = pytest.mark.gpu

DEV = "cuda"
TOL = {torch.float32: 1e-4, torch.float16: 5e-3, torch.bfloat16: 2e-2}
SCRATCH_BYTES = 2 << 20


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("shape", [(2, 32, 8, 128, 4096), (1, 64, 8, 128, 8192),
                                   (3, 16, 2, 64, 1000)])
def test_noalloc_matches_workspace_entry_point_twice(dtype, shape):
    B, Hq, Hkv, D, T = shape
    need = capi.lib().frn_gqa_decode_workspace_size(B, Hq, Hkv, D, T)
    if dtype == torch.float32:
        # fp32 never takes the tensor-core kernel; a non-zero need means the
        # context is split and the partials go through the static scratch.
        assert 0 < need <= SCRATCH_BYTES
    scale = 1.0 / math.sqrt(D)
    tol = TOL[dtype]
    for call in range(2):
        q, k, v = orc.make_gqa_inputs(B, Hq, Hkv, D, T, seed=100 + call, dtype=dtype)
        qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
        ref = capi.gqa_decode_attention(qd, kd, vd, scale)
        out = torch.full_like(qd, float("nan"))
        capi.gqa_decode_attention_noalloc(qd, kd, vd, scale, out)
        torch.cuda.synchronize()
        torch.testing.assert_close(out.float().cpu(), ref.float().cpu(), atol=tol, rtol=tol)
        torch.testing.assert_close(out.float().cpu(), orc.gqa_decode_reference(q, k, v, scale),
                                   atol=tol, rtol=tol)
    assert capi.device_error(0) == 0


def test_noalloc_bf16_needs_no_scratch_at_any_batch():
    """bf16 shapes are served without scratch, whatever the fp32 path would need."""
    B, Hq, Hkv, D, T = 64, 32, 8, 128, 256
    q, k, v = orc.make_gqa_inputs(B, Hq, Hkv, D, T, seed=7)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    out = torch.empty_like(qd)
    capi.gqa_decode_attention_noalloc(qd, kd, vd, 1.0 / math.sqrt(D), out)
    torch.cuda.synchronize()
    torch.testing.assert_close(out.float().cpu(),
                               orc.gqa_decode_reference(q, k, v, 1.0 / math.sqrt(D)),
                               atol=2e-2, rtol=2e-2)
