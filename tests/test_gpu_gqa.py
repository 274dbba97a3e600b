"""GPU parity of decode-step GQA attention (frn_gqa_decode_attention and the
gqa_attention_cuda / GQADecodeAttentionV2/V3 surface) against the fp64 CPU
oracle, with the context split across SMs (workspace) and without."""
import math

import pytest
import torch

from oracle import gqa_decode as orc
from src import capi

pytestmark = pytest.mark.gpu

DEV = "cuda"
TOL = {torch.float32: 1e-4, torch.float16: 5e-3, torch.bfloat16: 2e-2}

SHAPES = [
    # (B, Hq, Hkv, D, T)
    (1, 32, 8, 128, 1),
    (1, 32, 8, 128, 100),
    (2, 32, 8, 128, 4096),
    (4, 8, 8, 64, 777),
    (3, 16, 2, 64, 2048),
    (1, 64, 8, 128, 8192),
    # tensor-core path edges: context not a multiple of the 64-token stage,
    # shorter than a stage, G = 2, 3, 7, many batches
    (8, 32, 8, 128, 333),
    (2, 8, 4, 64, 64),
    (1, 12, 4, 128, 65),
    (16, 32, 8, 128, 512),
    (2, 28, 4, 128, 1000),
]


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("use_ws", [True, False])
def test_gqa_decode_bf16(shape, use_ws):
    B, Hq, Hkv, D, T = shape
    q, k, v = orc.make_gqa_inputs(B, Hq, Hkv, D, T, seed=T + Hq)
    scale = 1.0 / math.sqrt(D)
    out = capi.gqa_decode_attention(q.to(DEV), k.to(DEV), v.to(DEV), scale, use_workspace=use_ws)
    torch.cuda.synchronize()
    ref = orc.gqa_decode_reference(q, k, v, scale)
    torch.testing.assert_close(out.float().cpu(), ref, atol=TOL[q.dtype], rtol=TOL[q.dtype])


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
def test_gqa_decode_dtypes(dtype):
    B, Hq, Hkv, D, T = 2, 24, 4, 128, 1500
    q, k, v = orc.make_gqa_inputs(B, Hq, Hkv, D, T, seed=3, dtype=dtype)
    scale = 0.7 / math.sqrt(D)
    out = capi.gqa_decode_attention(q.to(DEV), k.to(DEV), v.to(DEV), scale)
    torch.cuda.synchronize()
    ref = orc.gqa_decode_reference(q, k, v, scale)
    torch.testing.assert_close(out.float().cpu(), ref, atol=TOL[dtype], rtol=TOL[dtype])


def test_gqa_modules_match_reference_surface():
    from src.gqa_attention_forward import (GQADecodeAttentionV2, GQADecodeAttentionV3,
                                           pytorch_gqa_decode_attention)
    from src.load_gqa_attention import gqa_attention_cuda

    B, Hq, Hkv, D, T = 2, 32, 8, 128, 640
    q, k, v = orc.make_gqa_inputs(B, Hq, Hkv, D, T, seed=11)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    ref = orc.gqa_decode_reference(q, k, v, 1.0 / math.sqrt(D))
    for mod in (GQADecodeAttentionV2(Hq, Hkv, D), GQADecodeAttentionV3(Hq, Hkv, D)):
        torch.testing.assert_close(mod(qd, kd, vd).float().cpu(), ref, atol=2e-2, rtol=2e-2)
    out = torch.empty_like(qd)
    gqa_attention_cuda.gqa_decode_v3(qd, kd, vd, out, Hq // Hkv, 1.0 / math.sqrt(D))
    torch.testing.assert_close(out.float().cpu(), ref, atol=2e-2, rtol=2e-2)
    torch.testing.assert_close(pytorch_gqa_decode_attention(qd.float(), kd.float(), vd.float(),
                                                            Hkv).cpu(), ref, atol=1e-4, rtol=1e-4)
    with pytest.raises(RuntimeError, match="group_size"):
        gqa_attention_cuda.gqa_decode_v3(qd, kd, vd, out, 3, 1.0)
    with pytest.raises(capi.FrnError, match="head_dim"):
        capi.gqa_decode_attention(qd[..., :96].contiguous(), kd[..., :96].contiguous(),
                                  vd[..., :96].contiguous(), 1.0)
    assert capi.device_error(0) == 0
