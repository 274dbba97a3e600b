"""ctypes binding of the C ABI in include/frn_b200.h.

This is the binding a non-torch host would write (a cgo or JNI host binds the
same symbols the same way); the parity tests use it to call libfrn_b200.so
exactly through its extern "C" entry points, passing raw device pointers,
element strides and the current CUDA stream.
"""

from __future__ import annotations

import ctypes
from ctypes import c_char_p, c_float, c_int, c_int64, c_size_t, c_uint32, c_void_p

from src._build import load_library

FRN_OK = 0
FRN_ERR_INVALID_ARGUMENT = 1
FRN_ERR_UNSUPPORTED = 2
FRN_ERR_MISALIGNED = 3
FRN_ERR_WORKSPACE = 4
FRN_ERR_CUDA = 5
FRN_ERR_DEVICE_TIMEOUT = 6

FRN_DTYPE_F32 = 0
FRN_DTYPE_F16 = 1
FRN_DTYPE_BF16 = 2

FRN_KERNEL_AUTO = 0
FRN_KERNEL_TILE_N128 = 1
FRN_KERNEL_TILE_N192 = 2
FRN_KERNEL_TILE_N256 = 3
FRN_KERNEL_DECODE = 4
FRN_KERNEL_PAIR_N128 = 5
FRN_KERNEL_PAIR_N160 = 6
FRN_KERNEL_PAIR_N192 = 7
FRN_KERNEL_PAIR_N224 = 8
FRN_KERNEL_PAIR_N256 = 9
FRN_KERNEL_PAIR_AUTO = 10
FRN_KERNEL_WIDE_N128 = 11
FRN_KERNEL_WIDE_N192 = 12
FRN_KERNEL_WIDE_N224 = 13
FRN_KERNEL_WIDE_N256 = 14
FRN_KERNEL_WIDE_N176 = 21

# name -> (restype, argtypes); must cover every function in include/frn_b200.h
class W8Linear(ctypes.Structure):
    """struct frn_w8_linear of include/frn_b200.h (one problem of a grouped
    int8 call)."""
    _fields_ = [("x", c_void_p), ("M", c_int64), ("K", c_int64), ("x_row_stride", c_int64),
                ("wq", c_void_p), ("N", c_int64), ("wq_row_stride", c_int64),
                ("w_scale", c_void_p), ("bias", c_void_p), ("out", c_void_p),
                ("out_row_stride", c_int64)]


PROTOTYPES = {
    "frn_abi_version": (c_int, []),
    "frn_last_error": (c_char_p, []),
    "frn_rmsnorm_normalize": (
        c_int,
        [c_int, c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_int64, c_int64,
         c_float, c_int, c_void_p],
    ),
    "frn_fused_rmsnorm_linear_workspace_size": (c_size_t, [c_int, c_int64, c_int64, c_int64]),
    "frn_fused_rmsnorm_linear": (
        c_int,
        [c_int, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int64, c_int64, c_void_p,
         c_float, c_void_p, c_int64, c_void_p, c_size_t, c_void_p],
    ),
    "frn_fused_rmsnorm_linear_ex": (
        c_int,
        [c_int, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int64, c_int64, c_void_p,
         c_float, c_void_p, c_int64, c_void_p, c_size_t, c_int, c_void_p],
    ),
    "frn_fused_rmsnorm_linear_w8": (
        c_int,
        [c_int, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int64, c_int64, c_void_p,
         c_void_p, c_float, c_void_p, c_int64, c_void_p],
    ),
    "frn_fused_rmsnorm_linear_w8_grouped": (
        c_int, [c_int, ctypes.POINTER(W8Linear), c_int, c_float, c_void_p]),
    "frn_quantize_int8_per_channel": (
        c_int,
        [c_int, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int64, c_void_p, c_void_p],
    ),
    "frn_fused_rmsnorm_linear_split": (
        c_int,
        [c_int, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int64, c_int64, c_void_p,
         c_float, c_int, ctypes.POINTER(c_int64), ctypes.POINTER(c_void_p),
         ctypes.POINTER(c_int64), c_void_p],
    ),
    "frn_rmsnorm_swiglu": (
        c_int,
        [c_int, c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64,
         c_int64, c_int64, c_float, c_int, c_void_p],
    ),
    "frn_fused_rmsnorm_swiglu": (
        c_int,
        [c_int, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int64, c_int64, c_void_p,
         c_float, c_void_p, c_int64, c_void_p],
    ),
    "frn_gqa_decode_workspace_size": (c_size_t, [c_int64, c_int64, c_int64, c_int64, c_int64]),
    "frn_gqa_decode_attention": (
        c_int,
        [c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64,
         c_int64, c_float, c_void_p, c_size_t, c_void_p],
    ),
    "frn_gqa_decode_attention_noalloc": (
        c_int,
        [c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64,
         c_int64, c_float, c_void_p],
    ),
    "frn_device_error": (c_int, [c_int, ctypes.POINTER(c_uint32), c_int]),
    "frn_selftest_wait_timeout": (c_int, [c_int, c_void_p]),
}

_lib = None


class FrnError(RuntimeError):
    def __init__(self, code: int, what: str, message: str):
        super().__init__(f"{what} failed (status {code}): {message}")
        self.code = code


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        handle = load_library()
        for name, (res, args) in PROTOTYPES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def last_error() -> str:
    return lib().frn_last_error().decode()


def check(rc: int, what: str) -> None:
    if rc != FRN_OK:
        raise FrnError(rc, what, last_error())


# ------------------------------------------------------------ torch helpers
def _dtype_code(t) -> int:
    import torch

    return {torch.float32: FRN_DTYPE_F32, torch.float16: FRN_DTYPE_F16,
            torch.bfloat16: FRN_DTYPE_BF16}[t.dtype]


def _stream_ptr(device) -> int:
    import torch

    return torch.cuda.current_stream(device).cuda_stream


def _on(device):
    """Makes `device` current for the call: every frn_* entry point works on
    the caller's current CUDA device (its SM count, its static scratch)."""
    import torch

    return torch.cuda.device(device)


def workspace_size(dtype_code: int, M: int, N: int, K: int) -> int:
    return int(lib().frn_fused_rmsnorm_linear_workspace_size(dtype_code, M, N, K))


def fused_rmsnorm_linear(x, w, bias=None, eps: float = 1e-6, out=None,
                         kernel: int = FRN_KERNEL_AUTO, workspace=None):
    """out = rsqrt(mean(x^2)+eps)[:,None] * (x @ w.T) + bias through the C ABI.

    x: [M, K] with unit inner stride (any 16B-legal row stride); w: [N, K].
    """
    import torch

    assert x.dim() == 2 and w.dim() == 2 and x.stride(1) == 1 and w.stride(1) == 1
    M, K = x.shape
    N = w.shape[0]
    if out is None:
        out = torch.empty(M, N, dtype=x.dtype, device=x.device)
    dt = _dtype_code(x)
    need = workspace_size(dt, M, N, K)
    if workspace is None and need > 0:
        workspace = torch.empty(need, dtype=torch.uint8, device=x.device)
    ws_ptr = workspace.data_ptr() if workspace is not None else None
    ws_bytes = workspace.numel() if workspace is not None else 0
    with _on(x.device):
        rc = lib().frn_fused_rmsnorm_linear_ex(
            dt, x.data_ptr(), M, K, x.stride(0), w.data_ptr(), N, w.stride(0),
            bias.data_ptr() if bias is not None else None, float(eps), out.data_ptr(),
            out.stride(0), ws_ptr, ws_bytes, int(kernel), _stream_ptr(x.device))
    check(rc, "frn_fused_rmsnorm_linear")
    return out


def rmsnorm_normalize(x, raw_output, b_new, h: int, eps: float, threads: int = 256):
    """In-place raw_output = raw_output * inv_rms(x) + b_new through the C ABI."""
    with _on(x.device):
        rc = lib().frn_rmsnorm_normalize(
            _dtype_code(x), x.data_ptr(), x.stride(0), raw_output.data_ptr(), raw_output.stride(0),
            b_new.data_ptr(), x.shape[0], h, raw_output.shape[1], float(eps), int(threads),
            _stream_ptr(x.device))
    check(rc, "frn_rmsnorm_normalize")
    return raw_output


def fused_rmsnorm_linear_w8(x, wq, w_scale, bias=None, eps: float = 1e-6, out=None):
    """out = inv_rms[:,None] * w_scale[None,:] * (x @ wq.T) + bias (int8 wq)."""
    import torch

    assert x.dim() == 2 and wq.dim() == 2 and x.stride(1) == 1 and wq.stride(1) == 1
    M, K = x.shape
    N = wq.shape[0]
    if out is None:
        out = torch.empty(M, N, dtype=x.dtype, device=x.device)
    with _on(x.device):
        rc = lib().frn_fused_rmsnorm_linear_w8(
            _dtype_code(x), x.data_ptr(), M, K, x.stride(0), wq.data_ptr(), N, wq.stride(0),
            w_scale.data_ptr(), bias.data_ptr() if bias is not None else None, float(eps),
            out.data_ptr(), out.stride(0), _stream_ptr(x.device))
    check(rc, "frn_fused_rmsnorm_linear_w8")
    return out


def fused_rmsnorm_linear_w8_grouped(problems, eps: float = 1e-6):
    """One launch for one or two independent int8 problems, each a tuple
    (x, wq, w_scale, bias, out) as in fused_rmsnorm_linear_w8 (out required);
    returns the outputs."""
    assert 1 <= len(problems) <= 2
    arr = (W8Linear * len(problems))()
    for a, (x, wq, w_scale, bias, out) in zip(arr, problems):
        assert x.dim() == 2 and wq.dim() == 2 and x.stride(1) == 1 and wq.stride(1) == 1
        assert x.device == problems[0][0].device and x.dtype == problems[0][0].dtype
        a.x, a.M, a.K, a.x_row_stride = x.data_ptr(), x.shape[0], x.shape[1], x.stride(0)
        a.wq, a.N, a.wq_row_stride = wq.data_ptr(), wq.shape[0], wq.stride(0)
        a.w_scale = w_scale.data_ptr()
        a.bias = bias.data_ptr() if bias is not None else None
        a.out, a.out_row_stride = out.data_ptr(), out.stride(0)
    x0 = problems[0][0]
    with _on(x0.device):
        rc = lib().frn_fused_rmsnorm_linear_w8_grouped(_dtype_code(x0), arr, len(problems),
                                                       float(eps), _stream_ptr(x0.device))
    check(rc, "frn_fused_rmsnorm_linear_w8_grouped")
    return [p[4] for p in problems]


def quantize_int8_per_channel(w):
    """(q int8 [N,K], scale fp32 [N]) of a weight on the GPU."""
    import torch

    N, K = w.shape
    q = torch.empty(N, K, dtype=torch.int8, device=w.device)
    scale = torch.empty(N, dtype=torch.float32, device=w.device)
    with _on(w.device):
        rc = lib().frn_quantize_int8_per_channel(_dtype_code(w), w.data_ptr(), N, K, w.stride(0),
                                                 q.data_ptr(), K, scale.data_ptr(),
                                                 _stream_ptr(w.device))
    check(rc, "frn_quantize_int8_per_channel")
    return q, scale


def fused_rmsnorm_linear_split(x, w, bias, eps: float, split_sizes, outs=None):
    """Fused RMSNorm -> Linear whose output columns land directly in
    len(split_sizes) separate [M, n_i] tensors (returned as a list)."""
    import torch

    assert x.dim() == 2 and w.dim() == 2 and x.stride(1) == 1 and w.stride(1) == 1
    M, K = x.shape
    N = w.shape[0]
    n = len(split_sizes)
    if outs is None:
        outs = [torch.empty(M, c, dtype=x.dtype, device=x.device) for c in split_sizes]
    cols = (c_int64 * n)(*[int(c) for c in split_sizes])
    ptrs = (c_void_p * n)(*[o.data_ptr() for o in outs])
    strides = (c_int64 * n)(*[o.stride(0) for o in outs])
    with _on(x.device):
        rc = lib().frn_fused_rmsnorm_linear_split(
            _dtype_code(x), x.data_ptr(), M, K, x.stride(0), w.data_ptr(), N, w.stride(0),
            bias.data_ptr() if bias is not None else None, float(eps), n, cols, ptrs, strides,
            _stream_ptr(x.device))
    check(rc, "frn_fused_rmsnorm_linear_split")
    return outs


def rmsnorm_swiglu(x, raw_output, output, b_new, h: int, intermediate: int, eps: float,
                   threads: int = 256):
    """output = silu(g * inv_rms + b_g) * (u * inv_rms + b_u) of a [gate | up]
    GEMM output, through the C ABI."""
    with _on(x.device):
        rc = lib().frn_rmsnorm_swiglu(
            _dtype_code(x), x.data_ptr(), x.stride(0), raw_output.data_ptr(), raw_output.stride(0),
            output.data_ptr(), output.stride(0), b_new.data_ptr(), x.shape[0], h, intermediate,
            float(eps), int(threads), _stream_ptr(x.device))
    check(rc, "frn_rmsnorm_swiglu")
    return output


def fused_rmsnorm_swiglu(x, w_combined, bias=None, eps: float = 1e-6, out=None):
    """One-launch RMSNorm -> [gate | up] projection -> SwiGLU through the C ABI.

    x: [M, K]; w_combined: [2I, K] (gate rows first); bias: [2I] or None;
    returns out [M, I]."""
    import torch

    assert x.dim() == 2 and w_combined.dim() == 2 and x.stride(1) == 1
    assert w_combined.stride(1) == 1 and w_combined.shape[0] % 2 == 0
    M, K = x.shape
    inter = w_combined.shape[0] // 2
    if out is None:
        out = torch.empty(M, inter, dtype=x.dtype, device=x.device)
    with _on(x.device):
        rc = lib().frn_fused_rmsnorm_swiglu(
            _dtype_code(x), x.data_ptr(), M, K, x.stride(0), w_combined.data_ptr(), inter,
            w_combined.stride(0), bias.data_ptr() if bias is not None else None, float(eps),
            out.data_ptr(), out.stride(0), _stream_ptr(x.device))
    check(rc, "frn_fused_rmsnorm_swiglu")
    return out


def gqa_decode_attention(q, k_cache, v_cache, scale: float, out=None, use_workspace=True):
    """Decode-step GQA attention through the C ABI: q [B, Hq, D], caches
    [B, T, Hkv, D] (contiguous); returns out [B, Hq, D]."""
    import torch

    B, Hq, D = q.shape
    T, Hkv = k_cache.shape[1], k_cache.shape[2]
    if out is None:
        out = torch.empty_like(q)
    with _on(q.device):
        ws_bytes = (int(lib().frn_gqa_decode_workspace_size(B, Hq, Hkv, D, T))
                    if use_workspace else 0)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device) if ws_bytes else None
    with _on(q.device):
        rc = lib().frn_gqa_decode_attention(
            _dtype_code(q), q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), out.data_ptr(),
            B, Hq, Hkv, D, T, float(scale), ws.data_ptr() if ws is not None else None, ws_bytes,
            _stream_ptr(q.device))
    check(rc, "frn_gqa_decode_attention")
    return out


def gqa_decode_attention_noalloc(q, k_cache, v_cache, scale: float, out):
    """frn_gqa_decode_attention_noalloc: the library's static scratch instead of
    a workspace; `out` must be preallocated (nothing is allocated here)."""
    B, Hq, D = q.shape
    T, Hkv = k_cache.shape[1], k_cache.shape[2]
    with _on(q.device):
        rc = lib().frn_gqa_decode_attention_noalloc(
            _dtype_code(q), q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), out.data_ptr(),
            B, Hq, Hkv, D, T, float(scale), _stream_ptr(q.device))
    check(rc, "frn_gqa_decode_attention_noalloc")
    return out


def selftest_wait_timeout(timeout_ms: int, stream=None) -> None:
    """Launch the bounded-wait self-test kernel (see include/frn_b200.h)."""
    check(lib().frn_selftest_wait_timeout(int(timeout_ms), stream), "frn_selftest_wait_timeout")


def device_error(device: int = 0, clear: bool = False) -> int:
    flags = c_uint32(0)
    check(lib().frn_device_error(device, ctypes.byref(flags), 1 if clear else 0),
          "frn_device_error")
    return int(flags.value)
