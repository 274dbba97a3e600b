"""``gqa_attention_cuda``: the decode-attention extension the reference loads
from src/load_gqa_attention.py.

Here the two exports (gqa_decode_v2, gqa_decode_v3; same arguments and
in-place output as the reference's csrc/gqa_attention.cpp:45-60) live in the
same in-tree ``denominator_cuda`` module as the fused RMSNorm ops, built for
sm_100a by src.load_cuda; this module only gives them the reference's name.
"""

from src.load_cuda import denominator_cuda as _ext


class _GqaAttentionModule:
    """Namespace with the reference module's two functions."""

    gqa_decode_v2 = staticmethod(_ext.gqa_decode_v2)
    gqa_decode_v3 = staticmethod(_ext.gqa_decode_v3)


gqa_attention_cuda = _GqaAttentionModule()
