// denominator.cpp -- the `denominator_cuda` Python module.
//
// Same module name and RMSNorm exports as the reference's pybind11 binding
// (reference csrc/denominator.cpp:152-213), re-implemented as a thin layer
// over the C ABI in include/frn_b200.h: tensors are checked the way the
// reference's host launchers check them (csrc/denominator_kernel.cu:1999-2001,
// same messages), then their pointers, row strides and the current CUDA stream
// are handed to libfrn_b200.so.  New exports: fused_rmsnorm_linear and
// fused_rmsnorm_swiglu (single-launch fused ops), the int8-weight path, and
// device_error.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "frn_b200.h"

namespace {

int dtype_code(const at::Tensor& t) {
  switch (t.scalar_type()) {
    case at::kFloat: return FRN_DTYPE_F32;
    case at::kHalf: return FRN_DTYPE_F16;
    case at::kBFloat16: return FRN_DTYPE_BF16;
    default: return -1;
  }
}

void check_rc(int rc, const char* what) {
  TORCH_CHECK(rc == FRN_OK, what, " failed (status ", rc, "): ", frn_last_error());
}

void* stream_of(const at::Tensor& t) {
  return static_cast<void*>(at::cuda::getCurrentCUDAStream(t.device().index()).stream());
}

void rmsnorm_normalize_impl(const at::Tensor& x, at::Tensor& raw_output, const at::Tensor& b_new,
                            int64_t h, double eps, int threads, const char* name) {
  TORCH_CHECK(x.dim() == 2, "x must be 2D");
  TORCH_CHECK(raw_output.dim() == 2, "raw_output must be 2D");
  TORCH_CHECK(x.is_cuda() && raw_output.is_cuda() && b_new.is_cuda(),
              "All tensors must be on CUDA");
  const int dt = dtype_code(x);
  TORCH_CHECK(dt >= 0, "Unsupported dtype for RMSNorm ", name,
              ": only fp32, fp16, bf16 supported");
  TORCH_CHECK(raw_output.scalar_type() == x.scalar_type() &&
                  b_new.scalar_type() == x.scalar_type(),
              "x, raw_output and b_new must share one dtype");
  TORCH_CHECK(x.size(0) == raw_output.size(0), "x and raw_output must have the same rows");
  TORCH_CHECK(h == x.size(1), "h (", h, ") must equal x.size(1) (", x.size(1), ")");
  TORCH_CHECK(b_new.numel() == raw_output.size(1), "b_new must have raw_output.size(1) elements");
  TORCH_CHECK(x.stride(1) == 1 || x.size(1) == 1, "x must have unit stride along its last dim");
  TORCH_CHECK(raw_output.stride(1) == 1 || raw_output.size(1) == 1,
              "raw_output must have unit stride along its last dim");
  const at::Tensor b = b_new.contiguous();
  const c10::cuda::CUDAGuard guard(x.device());
  check_rc(frn_rmsnorm_normalize(dt, x.data_ptr(), x.stride(0), raw_output.data_ptr(),
                                 raw_output.stride(0), b.data_ptr(), x.size(0), h,
                                 raw_output.size(1), static_cast<float>(eps), threads,
                                 stream_of(x)),
           name);
}

void rmsnorm_normalize(const at::Tensor& x, at::Tensor raw_output, const at::Tensor& b_new,
                       int64_t h, double eps) {
  rmsnorm_normalize_impl(x, raw_output, b_new, h, eps, 256, "rmsnorm_normalize");
}

void rmsnorm_normalize_512(const at::Tensor& x, at::Tensor raw_output, const at::Tensor& b_new,
                           int64_t h, double eps) {
  rmsnorm_normalize_impl(x, raw_output, b_new, h, eps, 512, "rmsnorm_normalize_512");
}

std::vector<at::Tensor> fused_rmsnorm_linear_split(const at::Tensor& x_in, const at::Tensor& w,
                                                   const c10::optional<at::Tensor>& b_new,
                                                   double eps, std::vector<int64_t> split_sizes) {
  TORCH_CHECK(x_in.dim() == 2 && w.dim() == 2, "x and W_fused must be 2D");
  TORCH_CHECK(x_in.is_cuda() && w.is_cuda() && (!b_new || b_new->is_cuda()),
              "All tensors must be on CUDA");
  TORCH_CHECK(x_in.scalar_type() == at::kBFloat16 || x_in.scalar_type() == at::kHalf,
              "fused_rmsnorm_linear_split supports bf16 and fp16 (got ", x_in.scalar_type(), ")");
  TORCH_CHECK(w.scalar_type() == x_in.scalar_type(), "x and W_fused must share one dtype");
  TORCH_CHECK(x_in.size(1) == w.size(1), "x.size(1) != W_fused.size(1)");
  const int n = static_cast<int>(split_sizes.size());
  TORCH_CHECK(n >= 1 && n <= FRN_MAX_PARTS, "split_sizes must have 1..", FRN_MAX_PARTS,
              " entries");
  const at::Tensor x = (x_in.stride(1) == 1 || x_in.size(1) == 1) ? x_in : x_in.contiguous();
  const at::Tensor wc = (w.stride(1) == 1) ? w : w.contiguous();
  const int64_t M = x.size(0), K = x.size(1), N = wc.size(0);
  at::Tensor b;
  const void* bptr = nullptr;
  if (b_new && b_new->defined()) {
    TORCH_CHECK(b_new->numel() == N && b_new->scalar_type() == x.scalar_type(),
                "b_new must have W_fused.size(0) elements of x's dtype");
    b = b_new->contiguous();
    bptr = b.data_ptr();
  }
  std::vector<at::Tensor> outs;
  int64_t cols[FRN_MAX_PARTS], strides[FRN_MAX_PARTS];
  void* ptrs[FRN_MAX_PARTS];
  for (int i = 0; i < n; ++i) {
    outs.push_back(at::empty({M, split_sizes[i]}, x.options()));
    cols[i] = split_sizes[i];
    strides[i] = outs.back().stride(0);
    ptrs[i] = outs.back().data_ptr();
  }
  const c10::cuda::CUDAGuard guard(x.device());
  check_rc(frn_fused_rmsnorm_linear_split(dtype_code(x), x.data_ptr(), M, K, x.stride(0),
                                          wc.data_ptr(), N, wc.stride(0), bptr,
                                          static_cast<float>(eps), n, cols, ptrs, strides,
                                          stream_of(x)),
           "fused_rmsnorm_linear_split");
  return outs;
}

// ---- decode-step GQA attention (gqa_attention_cuda exports of the reference)
void gqa_decode_impl(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                     at::Tensor& out, double scale, const char* name) {
  TORCH_CHECK(q.dim() == 3 && k.dim() == 4 && v.dim() == 4 && out.dim() == 3,
              name, ": q/out must be [batch, heads, head_dim], caches [batch, ctx, kv_heads, head_dim]");
  TORCH_CHECK(q.is_cuda() && k.is_cuda() && v.is_cuda() && out.is_cuda(),
              "All tensors must be on CUDA");
  const int dt = dtype_code(q);
  TORCH_CHECK(dt >= 0, name, ": only fp32, fp16, bf16 supported");
  TORCH_CHECK(k.scalar_type() == q.scalar_type() && v.scalar_type() == q.scalar_type() &&
                  out.scalar_type() == q.scalar_type(),
              name, ": q, caches and output must share one dtype");
  TORCH_CHECK(k.sizes() == v.sizes(), name, ": k_cache and v_cache shapes differ");
  TORCH_CHECK(out.sizes() == q.sizes(), name, ": output must match q");
  TORCH_CHECK(k.size(0) == q.size(0) && k.size(3) == q.size(2), name, ": batch/head_dim mismatch");
  TORCH_CHECK(q.is_contiguous() && k.is_contiguous() && v.is_contiguous() && out.is_contiguous(),
              name, ": tensors must be contiguous");
  const int64_t B = q.size(0), Hq = q.size(1), D = q.size(2), T = k.size(1), Hkv = k.size(2);
  const c10::cuda::CUDAGuard guard(q.device());
  const size_t ws_bytes = frn_gqa_decode_workspace_size(B, Hq, Hkv, D, T);
  at::Tensor ws;
  if (ws_bytes > 0) ws = at::empty({static_cast<int64_t>(ws_bytes)}, q.options().dtype(at::kByte));
  check_rc(frn_gqa_decode_attention(dt, q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                    B, Hq, Hkv, D, T, static_cast<float>(scale),
                                    ws_bytes ? ws.data_ptr() : nullptr, ws_bytes, stream_of(q)),
           name);
}

void gqa_decode_v2(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, at::Tensor out,
                   double scale) {
  gqa_decode_impl(q, k, v, out, scale, "gqa_decode_v2");
}

void gqa_decode_v3(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, at::Tensor out,
                   int64_t group_size, double scale) {
  TORCH_CHECK(k.dim() == 4 && group_size * k.size(2) == q.size(1),
              "gqa_decode_v3: group_size * num_kv_heads must equal num_q_heads");
  gqa_decode_impl(q, k, v, out, scale, "gqa_decode_v3");
}

void rmsnorm_swiglu_impl(const at::Tensor& x, const at::Tensor& raw_output, at::Tensor& output,
                         const at::Tensor& b_new, int64_t h, int64_t intermediate, double eps,
                         int threads, const char* name) {
  TORCH_CHECK(x.dim() == 2, "x must be 2D");
  TORCH_CHECK(raw_output.dim() == 2, "raw_output must be 2D");
  TORCH_CHECK(output.dim() == 2, "output must be 2D");
  TORCH_CHECK(x.is_cuda() && raw_output.is_cuda() && output.is_cuda() && b_new.is_cuda(),
              "All tensors must be on CUDA");
  const int dt = dtype_code(x);
  TORCH_CHECK(dt >= 0, "Unsupported dtype for RMSNorm SwiGLU: only fp32, fp16, bf16 supported");
  TORCH_CHECK(raw_output.scalar_type() == x.scalar_type() &&
                  output.scalar_type() == x.scalar_type() && b_new.scalar_type() == x.scalar_type(),
              "x, raw_output, output and b_new must share one dtype");
  TORCH_CHECK(raw_output.size(0) == x.size(0) && output.size(0) == x.size(0),
              "x, raw_output and output must have the same rows");
  TORCH_CHECK(h == x.size(1), "h (", h, ") must equal x.size(1) (", x.size(1), ")");
  TORCH_CHECK(raw_output.size(1) == 2 * intermediate, "raw_output must have 2*intermediate columns");
  TORCH_CHECK(output.size(1) == intermediate, "output must have intermediate columns");
  TORCH_CHECK(b_new.numel() == 2 * intermediate, "b_new must have 2*intermediate elements");
  TORCH_CHECK(x.stride(1) == 1 && raw_output.stride(1) == 1 && output.stride(1) == 1,
              "x, raw_output and output must have unit stride along their last dim");
  const at::Tensor b = b_new.contiguous();
  const c10::cuda::CUDAGuard guard(x.device());
  check_rc(frn_rmsnorm_swiglu(dt, x.data_ptr(), x.stride(0), raw_output.data_ptr(),
                              raw_output.stride(0), output.data_ptr(), output.stride(0),
                              b.data_ptr(), x.size(0), h, intermediate, static_cast<float>(eps),
                              threads, stream_of(x)),
           name);
}

void rmsnorm_swiglu(const at::Tensor& x, const at::Tensor& raw_output, at::Tensor output,
                    const at::Tensor& b_new, int64_t h, int64_t intermediate, double eps) {
  rmsnorm_swiglu_impl(x, raw_output, output, b_new, h, intermediate, eps, 256, "rmsnorm_swiglu");
}

void rmsnorm_swiglu_512(const at::Tensor& x, const at::Tensor& raw_output, at::Tensor output,
                        const at::Tensor& b_new, int64_t h, int64_t intermediate, double eps) {
  rmsnorm_swiglu_impl(x, raw_output, output, b_new, h, intermediate, eps, 512,
                      "rmsnorm_swiglu_512");
}

at::Tensor fused_rmsnorm_swiglu(const at::Tensor& x_in, const at::Tensor& w,
                                const c10::optional<at::Tensor>& b_combined, double eps,
                                c10::optional<at::Tensor> out) {
  TORCH_CHECK(x_in.dim() == 2, "x must be 2D");
  TORCH_CHECK(w.dim() == 2, "W_combined must be 2D");
  TORCH_CHECK(x_in.is_cuda() && w.is_cuda() && (!b_combined || b_combined->is_cuda()),
              "All tensors must be on CUDA");
  TORCH_CHECK(x_in.scalar_type() == at::kBFloat16 || x_in.scalar_type() == at::kHalf,
              "fused_rmsnorm_swiglu supports bf16 and fp16 (got ", x_in.scalar_type(), ")");
  TORCH_CHECK(w.scalar_type() == x_in.scalar_type(), "x and W_combined must share one dtype");
  TORCH_CHECK(x_in.size(1) == w.size(1), "x.size(1) (", x_in.size(1),
              ") != W_combined.size(1) (", w.size(1), ")");
  TORCH_CHECK(w.size(0) % 2 == 0, "W_combined must have 2*intermediate rows");
  TORCH_CHECK(x_in.device() == w.device(), "x and W_combined must be on the same device");
  const at::Tensor x = (x_in.stride(1) == 1 || x_in.size(1) == 1) ? x_in : x_in.contiguous();
  const at::Tensor wc = (w.stride(1) == 1) ? w : w.contiguous();
  const int64_t M = x.size(0), K = x.size(1), I = wc.size(0) / 2;
  at::Tensor b;
  const void* bptr = nullptr;
  if (b_combined && b_combined->defined()) {
    TORCH_CHECK(b_combined->scalar_type() == x.scalar_type(), "b_combined must share x's dtype");
    TORCH_CHECK(b_combined->numel() == 2 * I, "b_combined must have W_combined.size(0) elements");
    b = b_combined->contiguous();
    bptr = b.data_ptr();
  }
  at::Tensor o;
  if (out && out->defined()) {
    o = *out;
    TORCH_CHECK(o.dim() == 2 && o.size(0) == M && o.size(1) == I, "out must be [M, intermediate]");
    TORCH_CHECK(o.scalar_type() == x.scalar_type() && o.is_cuda(), "out dtype/device mismatch");
    TORCH_CHECK(o.stride(1) == 1, "out must have unit stride along its last dim");
  } else {
    o = at::empty({M, I}, x.options());
  }
  const c10::cuda::CUDAGuard guard(x.device());
  check_rc(frn_fused_rmsnorm_swiglu(dtype_code(x), x.data_ptr(), M, K, x.stride(0), wc.data_ptr(),
                                    I, wc.stride(0), bptr, static_cast<float>(eps), o.data_ptr(),
                                    o.stride(0), stream_of(x)),
           "fused_rmsnorm_swiglu");
  return o;
}

at::Tensor fused_rmsnorm_linear(const at::Tensor& x_in, const at::Tensor& w,
                                const c10::optional<at::Tensor>& b_new, double eps,
                                c10::optional<at::Tensor> out, int64_t kernel) {
  TORCH_CHECK(x_in.dim() == 2, "x must be 2D");
  TORCH_CHECK(w.dim() == 2, "W_fused must be 2D");
  TORCH_CHECK(x_in.is_cuda() && w.is_cuda() && (!b_new || b_new->is_cuda()),
              "All tensors must be on CUDA");
  TORCH_CHECK(x_in.scalar_type() == at::kBFloat16 || x_in.scalar_type() == at::kHalf,
              "fused_rmsnorm_linear supports bf16 and fp16 (got ", x_in.scalar_type(), ")");
  TORCH_CHECK(w.scalar_type() == x_in.scalar_type(), "x and W_fused must share one dtype");
  TORCH_CHECK(x_in.size(1) == w.size(1), "x.size(1) (", x_in.size(1), ") != W_fused.size(1) (",
              w.size(1), ")");
  TORCH_CHECK(x_in.device() == w.device(), "x and W_fused must be on the same device");
  // Keep strided row views (k_pass in DeepseekV3 attention); only a
  // non-unit inner stride forces a copy.
  const at::Tensor x = (x_in.stride(1) == 1 || x_in.size(1) == 1) ? x_in : x_in.contiguous();
  const at::Tensor wc = (w.stride(1) == 1) ? w : w.contiguous();
  const int64_t M = x.size(0), K = x.size(1), N = wc.size(0);
  at::Tensor b;
  const void* bptr = nullptr;
  if (b_new && b_new->defined()) {
    TORCH_CHECK(b_new->scalar_type() == x.scalar_type(), "b_new must share x's dtype");
    TORCH_CHECK(b_new->numel() == N, "b_new must have W_fused.size(0) elements");
    b = b_new->contiguous();
    bptr = b.data_ptr();
  }
  at::Tensor o;
  if (out && out->defined()) {
    o = *out;
    TORCH_CHECK(o.dim() == 2 && o.size(0) == M && o.size(1) == N, "out must be [M, N]");
    TORCH_CHECK(o.scalar_type() == x.scalar_type() && o.is_cuda(), "out dtype/device mismatch");
    TORCH_CHECK(o.stride(1) == 1, "out must have unit stride along its last dim");
  } else {
    o = at::empty({M, N}, x.options());
  }
  const c10::cuda::CUDAGuard guard(x.device());
  const int dt = dtype_code(x);
  const size_t ws_bytes = frn_fused_rmsnorm_linear_workspace_size(dt, M, N, K);
  at::Tensor ws;
  if (ws_bytes > 0)
    ws = at::empty({static_cast<int64_t>(ws_bytes)}, x.options().dtype(at::kByte));
  check_rc(frn_fused_rmsnorm_linear_ex(dt, x.data_ptr(), M, K, x.stride(0), wc.data_ptr(), N,
                                       wc.stride(0), bptr, static_cast<float>(eps), o.data_ptr(),
                                       o.stride(0), ws_bytes ? ws.data_ptr() : nullptr, ws_bytes,
                                       static_cast<int>(kernel), stream_of(x)),
           "fused_rmsnorm_linear");
  return o;
}

// Checks one int8 problem's tensors and fills its C-ABI descriptor; `keep`
// holds the contiguous copies (if any) alive until the launch.
static frn_w8_linear prepare_w8(const at::Tensor& x_in, const at::Tensor& qweight,
                                const at::Tensor& w_scale, const c10::optional<at::Tensor>& b_new,
                                const c10::optional<at::Tensor>& out, std::vector<at::Tensor>& keep) {
  TORCH_CHECK(x_in.dim() == 2 && qweight.dim() == 2, "x and qweight must be 2D");
  TORCH_CHECK(x_in.is_cuda() && qweight.is_cuda() && w_scale.is_cuda() &&
                  (!b_new || b_new->is_cuda()),
              "All tensors must be on CUDA");
  TORCH_CHECK(x_in.scalar_type() == at::kBFloat16 || x_in.scalar_type() == at::kHalf,
              "fused_rmsnorm_linear_w8 takes bf16 or fp16 x");
  TORCH_CHECK(qweight.scalar_type() == at::kChar, "qweight must be int8");
  TORCH_CHECK(w_scale.scalar_type() == at::kFloat && w_scale.numel() == qweight.size(0),
              "w_scale must be fp32 with qweight.size(0) elements");
  TORCH_CHECK(x_in.size(1) == qweight.size(1), "x.size(1) != qweight.size(1)");
  const at::Tensor x = (x_in.stride(1) == 1) ? x_in : x_in.contiguous();
  const at::Tensor q = qweight.stride(1) == 1 ? qweight : qweight.contiguous();
  const at::Tensor sc = w_scale.contiguous();
  const int64_t M = x.size(0), K = x.size(1), N = q.size(0);
  const void* bptr = nullptr;
  if (b_new && b_new->defined()) {
    TORCH_CHECK(b_new->scalar_type() == x.scalar_type() && b_new->numel() == N,
                "b_new must share x's dtype and have qweight.size(0) elements");
    keep.push_back(b_new->contiguous());
    bptr = keep.back().data_ptr();
  }
  at::Tensor o = (out && out->defined()) ? *out : at::empty({M, N}, x.options());
  TORCH_CHECK(o.dim() == 2 && o.size(0) == M && o.size(1) == N && o.stride(1) == 1,
              "out must be [M, N] with unit inner stride");
  keep.push_back(x);
  keep.push_back(q);
  keep.push_back(sc);
  keep.push_back(o);
  frn_w8_linear d;
  d.x = x.data_ptr();
  d.M = M;
  d.K = K;
  d.x_row_stride = x.stride(0);
  d.wq = static_cast<const int8_t*>(q.data_ptr());
  d.N = N;
  d.wq_row_stride = q.stride(0);
  d.w_scale = sc.data_ptr<float>();
  d.bias = bptr;
  d.out = o.data_ptr();
  d.out_row_stride = o.stride(0);
  return d;
}

at::Tensor fused_rmsnorm_linear_w8(const at::Tensor& x_in, const at::Tensor& qweight,
                                   const at::Tensor& w_scale, const c10::optional<at::Tensor>& b_new,
                                   double eps, c10::optional<at::Tensor> out) {
  std::vector<at::Tensor> keep;
  const frn_w8_linear d = prepare_w8(x_in, qweight, w_scale, b_new, out, keep);
  const at::Tensor& x = keep[keep.size() - 4];
  const c10::cuda::CUDAGuard guard(x.device());
  check_rc(frn_fused_rmsnorm_linear_w8(dtype_code(x), d.x, d.M, d.K, d.x_row_stride, d.wq, d.N,
                                       d.wq_row_stride, d.w_scale, d.bias,
                                       static_cast<float>(eps), d.out, d.out_row_stride,
                                       stream_of(x)),
           "fused_rmsnorm_linear_w8");
  return keep.back();
}

// Two independent int8 problems (e.g. a layer's q_b and kv_b) in one launch.
std::tuple<at::Tensor, at::Tensor> fused_rmsnorm_linear_w8_grouped(
    const at::Tensor& x_a, const at::Tensor& qweight_a, const at::Tensor& w_scale_a,
    const c10::optional<at::Tensor>& b_a, const at::Tensor& x_b, const at::Tensor& qweight_b,
    const at::Tensor& w_scale_b, const c10::optional<at::Tensor>& b_b, double eps,
    c10::optional<at::Tensor> out_a, c10::optional<at::Tensor> out_b) {
  TORCH_CHECK(x_a.scalar_type() == x_b.scalar_type() && x_a.device() == x_b.device(),
              "grouped problems must share x's dtype and device");
  std::vector<at::Tensor> keep_a, keep_b;
  frn_w8_linear d[2];
  d[0] = prepare_w8(x_a, qweight_a, w_scale_a, b_a, out_a, keep_a);
  d[1] = prepare_w8(x_b, qweight_b, w_scale_b, b_b, out_b, keep_b);
  const c10::cuda::CUDAGuard guard(x_a.device());
  check_rc(frn_fused_rmsnorm_linear_w8_grouped(dtype_code(x_a), d, 2, static_cast<float>(eps),
                                               stream_of(x_a)),
           "fused_rmsnorm_linear_w8_grouped");
  return {keep_a.back(), keep_b.back()};
}

std::tuple<at::Tensor, at::Tensor> quantize_int8_per_channel(const at::Tensor& w_in) {
  TORCH_CHECK(w_in.dim() == 2, "weight must be 2D");
  TORCH_CHECK(w_in.is_cuda(), "All tensors must be on CUDA");
  const int dt = dtype_code(w_in);
  TORCH_CHECK(dt >= 0, "weight must be fp32, fp16 or bf16");
  const at::Tensor w = w_in.stride(1) == 1 ? w_in : w_in.contiguous();
  const int64_t N = w.size(0), K = w.size(1);
  at::Tensor q = at::empty({N, K}, w.options().dtype(at::kChar));
  at::Tensor sc = at::empty({N}, w.options().dtype(at::kFloat));
  const c10::cuda::CUDAGuard guard(w.device());
  check_rc(frn_quantize_int8_per_channel(dt, w.data_ptr(), N, K, w.stride(0),
                                         static_cast<int8_t*>(q.data_ptr()), K,
                                         sc.data_ptr<float>(), stream_of(w)),
           "quantize_int8_per_channel");
  return {q, sc};
}

int64_t device_error(int64_t device, bool clear) {
  uint32_t flags = 0;
  check_rc(frn_device_error(static_cast<int>(device), &flags, clear ? 1 : 0), "device_error");
  return static_cast<int64_t>(flags);
}

[[noreturn]] void out_of_scope(const char* name) {
  TORCH_CHECK(false, name,
              " belongs to the reference's LayerNorm (OPT) path, which this sm_100a build does "
              "not implement; use the RMSNorm exports");
}

at::Tensor compute_denominator(const at::Tensor&, c10::optional<int64_t>) {
  out_of_scope("compute_denominator");
}
void denominator_normalize(const at::Tensor&, at::Tensor, const at::Tensor&, int64_t, double) {
  out_of_scope("denominator_normalize");
}
at::Tensor compute_denominator_welford(const at::Tensor&, c10::optional<int64_t>) {
  out_of_scope("compute_denominator_welford");
}
void denominator_normalize_welford_512(const at::Tensor&, at::Tensor, const at::Tensor&, int64_t,
                                       double) {
  out_of_scope("denominator_normalize_welford_512");
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "B200 (sm_100a) fused RMSNorm -> Linear; RMSNorm exports of the reference module";
  m.def("rmsnorm_normalize", &rmsnorm_normalize,
        "In-place RMSNorm rescale of a GEMM output (256 threads per row)", py::arg("x"),
        py::arg("raw_output"), py::arg("b_new"), py::arg("h"), py::arg("eps"));
  m.def("rmsnorm_normalize_512", &rmsnorm_normalize_512,
        "In-place RMSNorm rescale of a GEMM output (512 threads per row)", py::arg("x"),
        py::arg("raw_output"), py::arg("b_new"), py::arg("h"), py::arg("eps"));
  m.def("fused_rmsnorm_linear_split", &fused_rmsnorm_linear_split,
        "fused_rmsnorm_linear whose output columns are written into separate [M, n_i] tensors",
        py::arg("x"), py::arg("W_fused"), py::arg("b_new"), py::arg("eps"),
        py::arg("split_sizes"));
  m.def("gqa_decode_v2", &gqa_decode_v2,
        "Decode-step GQA attention into output (context split across SMs)", py::arg("q"),
        py::arg("k_cache"), py::arg("v_cache"), py::arg("output"), py::arg("scale"));
  m.def("gqa_decode_v3", &gqa_decode_v3,
        "Decode-step GQA attention into output (context split across SMs)", py::arg("q"),
        py::arg("k_cache"), py::arg("v_cache"), py::arg("output"), py::arg("group_size"),
        py::arg("scale"));
  m.def("rmsnorm_swiglu", &rmsnorm_swiglu,
        "RMSNorm + SwiGLU of a [gate | up] GEMM output into output (256 threads per row)",
        py::arg("x"), py::arg("raw_output"), py::arg("output"), py::arg("b_new"), py::arg("h"),
        py::arg("intermediate"), py::arg("eps"));
  m.def("rmsnorm_swiglu_512", &rmsnorm_swiglu_512,
        "RMSNorm + SwiGLU of a [gate | up] GEMM output into output (512 threads per row)",
        py::arg("x"), py::arg("raw_output"), py::arg("output"), py::arg("b_new"), py::arg("h"),
        py::arg("intermediate"), py::arg("eps"));
  m.def("fused_rmsnorm_swiglu", &fused_rmsnorm_swiglu,
        "silu(r * (x @ Wg.T) + bg) * (r * (x @ Wu.T) + bu), r = rsqrt(mean(x^2)+eps); one launch",
        py::arg("x"), py::arg("W_combined"), py::arg("b_combined") = py::none(),
        py::arg("eps") = 1e-6, py::arg("out") = py::none());
  m.def("fused_rmsnorm_linear", &fused_rmsnorm_linear,
        "out = rsqrt(mean(x^2)+eps)[:,None] * (x @ W_fused.T) + b_new, one tcgen05 launch",
        py::arg("x"), py::arg("W_fused"), py::arg("b_new") = py::none(), py::arg("eps") = 1e-6,
        py::arg("out") = py::none(), py::arg("kernel") = 0);
  m.def("fused_rmsnorm_linear_w8", &fused_rmsnorm_linear_w8,
        "int8 weights: rsqrt(mean(x^2)+eps)[:,None] * w_scale * (x @ qweight.T) + b_new",
        py::arg("x"), py::arg("qweight"), py::arg("w_scale"), py::arg("b_new") = py::none(),
        py::arg("eps") = 1e-6, py::arg("out") = py::none());
  m.def("fused_rmsnorm_linear_w8_grouped", &fused_rmsnorm_linear_w8_grouped,
        "two independent int8 fused RMSNorm -> Linear problems in one launch",
        py::arg("x_a"), py::arg("qweight_a"), py::arg("w_scale_a"), py::arg("b_a"),
        py::arg("x_b"), py::arg("qweight_b"), py::arg("w_scale_b"), py::arg("b_b"),
        py::arg("eps") = 1e-6, py::arg("out_a") = py::none(), py::arg("out_b") = py::none());
  m.def("quantize_int8_per_channel", &quantize_int8_per_channel,
        "Symmetric per-output-channel int8 quantization on the GPU -> (qweight, w_scale)",
        py::arg("weight"));
  m.def("device_error", &device_error, "Read (and optionally clear) the device error word",
        py::arg("device") = 0, py::arg("clear") = false);
  m.def("compute_denominator", &compute_denominator, "LayerNorm path: not implemented",
        py::arg("x"), py::arg("stream_ptr") = py::none());
  m.def("denominator_normalize", &denominator_normalize, "LayerNorm path: not implemented",
        py::arg("x"), py::arg("raw_output"), py::arg("b_new"), py::arg("h"), py::arg("eps"));
  m.def("compute_denominator_welford", &compute_denominator_welford,
        "LayerNorm path: not implemented", py::arg("x"), py::arg("stream_ptr") = py::none());
  m.def("denominator_normalize_welford_512", &denominator_normalize_welford_512,
        "LayerNorm path: not implemented", py::arg("x"), py::arg("raw_output"), py::arg("b_new"),
        py::arg("h"), py::arg("eps"));
}
