"""The allocation-free GQA decode entry point (frn_gqa_decode_attention_noalloc),
called through the C ABI: two calls in a row, each checked against the
allocating entry point (frn_gqa_decode_attention with its workspace) within
the bf16 tolerance the GPU tests use.  Kept in a file collected last so it
also runs after every other GPU test in the same process."""
import math

import pytest
import torch

from oracle import gqa_decode as orc
from src import capi

pytestmark = pytest.mark.gpu

DEV = "cuda"
ATOL = RTOL = 2e-2


def test_noalloc_matches_workspace_entry_point_twice():
    # 2 x 32 heads over a 4096-token context uses the split path, i.e. the scratch.
    B, Hq, Hkv, D, T = 2, 32, 8, 128, 4096
    need = capi.lib().frn_gqa_decode_workspace_size(B, Hq, Hkv, D, T)
    assert 0 < need <= 2 << 20
    scale = 1.0 / math.sqrt(D)
    for call in range(2):
        q, k, v = orc.make_gqa_inputs(B, Hq, Hkv, D, T, seed=100 + call)
        qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
        ref = capi.gqa_decode_attention(qd, kd, vd, scale)
        out = torch.empty_like(qd)
        capi.gqa_decode_attention_noalloc(qd, kd, vd, scale, out)
        torch.cuda.synchronize()
        torch.testing.assert_close(out.float().cpu(), ref.float().cpu(), atol=ATOL, rtol=RTOL)
        torch.testing.assert_close(out.float().cpu(), orc.gqa_decode_reference(q, k, v, scale),
                                   atol=ATOL, rtol=RTOL)
