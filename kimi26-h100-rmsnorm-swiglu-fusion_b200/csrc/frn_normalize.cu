// frn_normalize.cu -- standalone RMSNorm epilogues of a precomputed GEMM
// output, kept for drop-in compatibility with the reference's
// `rmsnorm_normalize` / `_512` and `rmsnorm_swiglu` / `_512` exports
// (reference csrc/denominator_kernel.cu:856-1775, launched at :1947-2134).
// The in-place rescale:
//
//     inv_rms[r]       = rsqrt(sum_k x[r,k]^2 / h + eps)
//     raw_output[r, c] = round(raw_output[r, c] * inv_rms[r] + b_new[c])
//
// One CTA per row (256 or 512 threads, as the reference's V1 / V3).  The
// fused GEMM does not use this kernel; it is what a caller that already has
// a raw GEMM output (e.g. an fp32 cuBLAS result) applies afterwards.
// Differences from the reference, all deliberate: the row strides of x and
// raw_output are honoured (the reference indexes x + row*h), 16-byte vector
// access is used only when pointers and strides allow it, and rsqrtf
// replaces 1/sqrtf under --use_fast_math.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "frn_internal.h"

namespace frn {

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}

template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

template <typename T, int THREADS>
__global__ void __launch_bounds__(THREADS)
    rmsnorm_normalize_kernel(const T* __restrict__ x, int64_t xs, T* __restrict__ out,
                             int64_t os, const T* __restrict__ b, int h, int n, float eps,
                             int vec_x, int vec_o) {
  constexpr int V = 16 / sizeof(T);  // elements per 16-byte vector
  constexpr int WARPS = THREADS / 32;
  __shared__ float red[WARPS];
  __shared__ float inv_rms_s;
  const int64_t row = blockIdx.x;
  const T* xr = x + row * xs;
  T* orow = out + row * os;

  float ss = 0.f;
  if (vec_x) {
    const uint4* xv = reinterpret_cast<const uint4*>(xr);
    for (int i = threadIdx.x; i < h / V; i += THREADS) {
      uint4 u = xv[i];
      const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int j = 0; j < V; ++j) {
        const float f = to_f<T>(e[j]);
        ss = fmaf(f, f, ss);
      }
    }
  } else {
    for (int i = threadIdx.x; i < h; i += THREADS) {
      const float f = to_f<T>(xr[i]);
      ss = fmaf(f, f, ss);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < WARPS ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (threadIdx.x == 0) inv_rms_s = rsqrtf(v / static_cast<float>(h) + eps);
  }
  __syncthreads();
  const float inv_rms = inv_rms_s;

  if (vec_o) {
    uint4* ov = reinterpret_cast<uint4*>(orow);
    const uint4* bv = reinterpret_cast<const uint4*>(b);
    for (int i = threadIdx.x; i < n / V; i += THREADS) {
      uint4 u = ov[i];
      const uint4 bb = bv[i];
      T* e = reinterpret_cast<T*>(&u);
      const T* be = reinterpret_cast<const T*>(&bb);
#pragma unroll
      for (int j = 0; j < V; ++j) e[j] = from_f<T>(fmaf(to_f<T>(e[j]), inv_rms, to_f<T>(be[j])));
      ov[i] = u;
    }
  } else {
    for (int i = threadIdx.x; i < n; i += THREADS)
      orow[i] = from_f<T>(fmaf(to_f<T>(orow[i]), inv_rms, to_f<T>(b[i])));
  }
}

// RMSNorm + SwiGLU applied to a precomputed [gate | up] GEMM output
// (reference rmsnorm_swiglu_*_kernel, csrc/denominator_kernel.cu:1275-1775):
//     g = raw[r, c] * inv_rms + b[c],  u = raw[r, I + c] * inv_rms + b[I + c]
//     out[r, c] = round(g / (1 + exp(-g)) * u)                  (c < I)
template <typename T, int THREADS>
__global__ void __launch_bounds__(THREADS)
    rmsnorm_swiglu_kernel(const T* __restrict__ x, int64_t xs, const T* __restrict__ raw,
                          int64_t rs, T* __restrict__ out, int64_t os, const T* __restrict__ b,
                          int h, int inter, float eps, int vec_x, int vec_o) {
  constexpr int V = 16 / sizeof(T);
  constexpr int WARPS = THREADS / 32;
  __shared__ float red[WARPS];
  __shared__ float inv_rms_s;
  const int64_t row = blockIdx.x;
  const T* xr = x + row * xs;
  const T* gr = raw + row * rs;
  const T* ur = gr + inter;
  T* orow = out + row * os;

  float ss = 0.f;
  if (vec_x) {
    const uint4* xv = reinterpret_cast<const uint4*>(xr);
    for (int i = threadIdx.x; i < h / V; i += THREADS) {
      uint4 u = xv[i];
      const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int j = 0; j < V; ++j) {
        const float f = to_f<T>(e[j]);
        ss = fmaf(f, f, ss);
      }
    }
  } else {
    for (int i = threadIdx.x; i < h; i += THREADS) {
      const float f = to_f<T>(xr[i]);
      ss = fmaf(f, f, ss);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < WARPS ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (threadIdx.x == 0) inv_rms_s = rsqrtf(v / static_cast<float>(h) + eps);
  }
  __syncthreads();
  const float inv_rms = inv_rms_s;
  auto swiglu = [&](float g, float u, float bg, float bu) {
    const float gv = fmaf(g, inv_rms, bg), uv = fmaf(u, inv_rms, bu);
    return gv / (1.0f + expf(-gv)) * uv;
  };
  if (vec_o) {
    const uint4* gv4 = reinterpret_cast<const uint4*>(gr);
    const uint4* uv4 = reinterpret_cast<const uint4*>(ur);
    const uint4* bg4 = reinterpret_cast<const uint4*>(b);
    const uint4* bu4 = reinterpret_cast<const uint4*>(b + inter);
    uint4* ov = reinterpret_cast<uint4*>(orow);
    for (int i = threadIdx.x; i < inter / V; i += THREADS) {
      const uint4 g = gv4[i], u = uv4[i], bg = bg4[i], bu = bu4[i];
      uint4 o;
      const T* ge = reinterpret_cast<const T*>(&g);
      const T* ue = reinterpret_cast<const T*>(&u);
      const T* bge = reinterpret_cast<const T*>(&bg);
      const T* bue = reinterpret_cast<const T*>(&bu);
      T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
      for (int j = 0; j < V; ++j)
        oe[j] = from_f<T>(swiglu(to_f<T>(ge[j]), to_f<T>(ue[j]), to_f<T>(bge[j]), to_f<T>(bue[j])));
      ov[i] = o;
    }
  } else {
    for (int i = threadIdx.x; i < inter; i += THREADS)
      orow[i] = from_f<T>(swiglu(to_f<T>(gr[i]), to_f<T>(ur[i]), to_f<T>(b[i]),
                                 to_f<T>(b[inter + i])));
  }
}

template <typename T>
static int launch_swiglu_norm(const void* x, int64_t xs, const void* raw, int64_t rs, void* out,
                              int64_t os, const void* b, int64_t rows, int64_t h, int64_t inter,
                              float eps, int threads, cudaStream_t s) {
  constexpr int V = 16 / sizeof(T);
  auto aligned = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  const int vec_x = aligned(x) && (xs % V == 0) && (h % V == 0);
  const int vec_o = aligned(raw) && aligned(out) && aligned(b) && (rs % V == 0) &&
                    (os % V == 0) && (inter % V == 0);
  const T* xp = static_cast<const T*>(x);
  const T* rp = static_cast<const T*>(raw);
  T* op = static_cast<T*>(out);
  const T* bp = static_cast<const T*>(b);
  const dim3 grid(static_cast<unsigned>(rows));
  if (threads == 512)
    rmsnorm_swiglu_kernel<T, 512><<<grid, 512, 0, s>>>(xp, xs, rp, rs, op, os, bp, (int)h,
                                                       (int)inter, eps, vec_x, vec_o);
  else
    rmsnorm_swiglu_kernel<T, 256><<<grid, 256, 0, s>>>(xp, xs, rp, rs, op, os, bp, (int)h,
                                                       (int)inter, eps, vec_x, vec_o);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error("launch rmsnorm_swiglu", e);
  return 0;
}

int run_rmsnorm_swiglu(int dtype, const void* x, int64_t xs, const void* raw, int64_t rs,
                       void* out, int64_t os, const void* b, int64_t rows, int64_t h,
                       int64_t inter, float eps, int threads, cudaStream_t s) {
  switch (dtype) {
    case FRN_DTYPE_F32:
      return launch_swiglu_norm<float>(x, xs, raw, rs, out, os, b, rows, h, inter, eps, threads, s);
    case FRN_DTYPE_F16:
      return launch_swiglu_norm<__half>(x, xs, raw, rs, out, os, b, rows, h, inter, eps, threads, s);
    case FRN_DTYPE_BF16:
      return launch_swiglu_norm<__nv_bfloat16>(x, xs, raw, rs, out, os, b, rows, h, inter, eps,
                                               threads, s);
    default:
      return set_error(FRN_ERR_UNSUPPORTED,
                       "Unsupported dtype for RMSNorm SwiGLU: only fp32, fp16, bf16 supported");
  }
}

template <typename T>
static int launch_norm(const void* x, int64_t xs, void* out, int64_t os, const void* b,
                       int64_t rows, int64_t h, int64_t n, float eps, int threads,
                       cudaStream_t s) {
  constexpr int V = 16 / sizeof(T);
  auto aligned = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  const int vec_x = aligned(x) && (xs % V == 0) && (h % V == 0);
  const int vec_o = aligned(out) && aligned(b) && (os % V == 0) && (n % V == 0);
  const T* xp = static_cast<const T*>(x);
  T* op = static_cast<T*>(out);
  const T* bp = static_cast<const T*>(b);
  const dim3 grid(static_cast<unsigned>(rows));
  if (threads == 512)
    rmsnorm_normalize_kernel<T, 512><<<grid, 512, 0, s>>>(xp, xs, op, os, bp, (int)h, (int)n,
                                                          eps, vec_x, vec_o);
  else
    rmsnorm_normalize_kernel<T, 256><<<grid, 256, 0, s>>>(xp, xs, op, os, bp, (int)h, (int)n,
                                                          eps, vec_x, vec_o);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error("launch rmsnorm_normalize", e);
  return 0;
}

int run_rmsnorm_normalize(int dtype, const void* x, int64_t xs, void* out, int64_t os,
                          const void* b, int64_t rows, int64_t h, int64_t n, float eps,
                          int threads, cudaStream_t s) {
  switch (dtype) {
    case FRN_DTYPE_F32: return launch_norm<float>(x, xs, out, os, b, rows, h, n, eps, threads, s);
    case FRN_DTYPE_F16: return launch_norm<__half>(x, xs, out, os, b, rows, h, n, eps, threads, s);
    case FRN_DTYPE_BF16:
      return launch_norm<__nv_bfloat16>(x, xs, out, os, b, rows, h, n, eps, threads, s);
    default:
      return set_error(FRN_ERR_UNSUPPORTED,
                       "Unsupported dtype for RMSNorm normalize: only fp32, fp16, bf16 supported");
  }
}

}  // namespace frn
