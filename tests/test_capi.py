"""The C ABI library loads, exports every symbol include/frn_b200.h declares,
and its host-side validation rejects bad arguments before touching a GPU."""
import ctypes
import os
import re

import pytest

from src import capi

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include",
                      "frn_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(frn_[a-z0-9_]+)\s*\(", text)))


def test_every_declared_symbol_is_exported():
    lib = capi.lib()
    names = declared_functions()
    assert names, "no declarations parsed"
    for n in names:
        assert hasattr(lib, n), f"{n} missing from libfrn_b200.so"
    assert set(names) == set(capi.PROTOTYPES), "capi.PROTOTYPES out of sync with the header"


def test_header_constants_match_binding():
    text = open(HEADER).read()
    for name, value in re.findall(r"#define\s+(FRN_[A-Z0-9_]+)\s+(\d+)\b", text):
        if hasattr(capi, name):
            assert getattr(capi, name) == int(value), name


def test_abi_version_and_error_string():
    lib = capi.lib()
    assert lib.frn_abi_version() == 1
    assert isinstance(lib.frn_last_error(), bytes)


def _call(dtype=capi.FRN_DTYPE_BF16, M=4, K=64, xs=64, N=64, ws=64, os_=64, x=16, w=16, out=16,
          bias=None, kernel=0):
    return capi.lib().frn_fused_rmsnorm_linear_ex(dtype, x, M, K, xs, w, N, ws, bias, 1e-5, out,
                                                 os_, None, 0, kernel, None)


@pytest.mark.parametrize("kwargs,code", [
    (dict(dtype=capi.FRN_DTYPE_F32), capi.FRN_ERR_UNSUPPORTED),
    (dict(dtype=7), capi.FRN_ERR_UNSUPPORTED),
    (dict(K=0), capi.FRN_ERR_INVALID_ARGUMENT),
    (dict(N=-1), capi.FRN_ERR_INVALID_ARGUMENT),
    (dict(xs=32), capi.FRN_ERR_INVALID_ARGUMENT),
    (dict(K=60, xs=64), capi.FRN_ERR_MISALIGNED),
    (dict(N=60, os_=64), capi.FRN_ERR_MISALIGNED),
    (dict(xs=68), capi.FRN_ERR_MISALIGNED),
    (dict(x=24), capi.FRN_ERR_MISALIGNED),
    (dict(bias=40), capi.FRN_ERR_MISALIGNED),
    (dict(x=None), capi.FRN_ERR_INVALID_ARGUMENT),
])
def test_fused_linear_rejects_bad_arguments(kwargs, code):
    rc = _call(**kwargs)
    assert rc == code
    assert capi.last_error() != ""


def test_empty_batch_is_a_no_op():
    assert _call(M=0, x=None, out=None) == capi.FRN_OK


def test_normalize_validation():
    lib = capi.lib()
    f = lib.frn_rmsnorm_normalize
    assert f(9, 16, 8, 16, 8, 16, 2, 8, 8, 1e-5, 256, None) == capi.FRN_ERR_UNSUPPORTED
    assert f(2, 16, 8, 16, 8, 16, 2, 8, 8, 1e-5, 300, None) == capi.FRN_ERR_INVALID_ARGUMENT
    assert f(2, 16, 4, 16, 8, 16, 2, 8, 8, 1e-5, 256, None) == capi.FRN_ERR_INVALID_ARGUMENT
    assert f(2, None, 8, None, 8, None, 0, 8, 8, 1e-5, 512, None) == capi.FRN_OK


def test_workspace_query_is_host_only():
    assert capi.workspace_size(capi.FRN_DTYPE_BF16, 512, 12288, 1536) >= 0


def test_build_stamp_is_relocatable_and_covers_every_header():
    """The library's freshness stamp must not depend on where the tree sits
    (a copy on another machine would otherwise rebuild, and several ranks of
    one job would rebuild at once), and must cover every header the kernels
    include."""
    from src import _build

    assert _build.REPO_DIR not in _build._flags_key()
    csrc = _build.CSRC_DIR
    headers = {f for f in os.listdir(csrc) if f.endswith((".cuh", ".h"))}
    assert headers <= set(_build.HEADERS), headers - set(_build.HEADERS)
    sources = {f for f in os.listdir(csrc) if f.endswith(".cu")}
    assert sources == set(_build.CU_SOURCES)


def test_gqa_workspace_fits_the_static_scratch_on_b200():
    """With G <= 8 and head_dim <= 128 the split rule (about three CTAs per SM
    over batch x KV heads) keeps the fp32 split path's workspace under the
    2 MiB static scratch of frn_gqa_decode_attention_noalloc on a 148-SM part,
    so that entry point rejects no valid shape there.  Host-only query."""
    f = capi.lib().frn_gqa_decode_workspace_size
    worst = 0
    for B in (1, 2, 3, 4, 7, 16, 64, 300):
        for Hkv in (1, 2, 4, 8, 32):
            for G in (1, 2, 4, 8):
                for D in (64, 128):
                    for T in (1, 33, 1000, 8192, 131072):
                        worst = max(worst, f(B, Hkv * G, Hkv, D, T))
    assert 0 < worst <= 3 * 148 * 8 * (128 + 2) * 4 <= 2 << 20
