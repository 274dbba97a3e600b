// frn_gqa_decode.cu -- single-token (decode) grouped-query attention.
//
//   out[b, h, :] = softmax_t(scale * q[b, h, :] . K[b, t, h / G, :]) @ V[b, :, h / G, :]
//
// q [B, Hq, D], K/V caches [B, T, Hkv, D], out [B, Hq, D], all contiguous;
// G = Hq / Hkv query heads share one KV head.  Same contract as the
// reference's gqa_decode_v2 / gqa_decode_v3 (csrc/gqa_attention_kernel.cu),
// which run one block per (batch, head) or per (batch, KV head) over the whole
// context; with B * Hkv of a decode step (8 for Llama-3-8B at batch 1) that
// leaves most of the 148 SMs idle, so this kernel splits the context as well
// (flash-decoding):
//
//   pass 1  CTA (kv head, batch, split) streams its slice of K/V once for all
//           G query heads: each warp takes every 4th token, lanes hold D/32
//           elements of q, k, v; scores are reduced with warp shuffles and an
//           online softmax (base 2, q pre-scaled by scale * log2 e) keeps
//           (max, sum, acc[D]) per query head; the four warps merge in shared
//           memory.  With one split the CTA writes out directly, otherwise
//           it writes its (acc, max, sum) to the workspace.
//   pass 2  one CTA per (batch, head) merges the splits (rescaled by their
//           maxima) and writes out.
//
// The K/V stream is the cost (2 * B * T * Hkv * D elements); the split count
// is chosen so that about four CTAs per SM read it, each warp keeping a run of
// 8 K and 8 V rows in flight.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cfloat>
#include <cstdint>
#include <mutex>

#include "frn_internal.h"

namespace frn {

// Scratch for frn_gqa_decode_attention_noalloc: the split partials of one
// call live here instead of in a caller-allocated workspace.  Shared by every
// call in the process on a given device; nothing in it needs to start at zero
// (each call writes every slot it reads).
constexpr size_t kGqaNoAllocScratchBytes = size_t(2) << 20;  // 2 MiB
static __device__ __align__(256) unsigned char g_gqa_noalloc_scratch[kGqaNoAllocScratchBytes];

struct GqaParams {
  const void* q;
  const void* k;
  const void* v;
  void* out;
  float* ws_acc;  // [B*Hq*S*D] split partial accumulators (S > 1)
  float* ws_ml;   // [B*Hq*S*2] split (max, sum)
  int32_t B, Hq, Hkv, T, G, S, tokens_per_split;
  float qscale;   // scale * log2(e)
};

template <typename T, int E>
__device__ __forceinline__ void load_e(const T* p, float (&f)[E]);

template <>
__device__ __forceinline__ void load_e<float, 4>(const float* p, float (&f)[4]) {
  const float4 v = *reinterpret_cast<const float4*>(p);
  f[0] = v.x; f[1] = v.y; f[2] = v.z; f[3] = v.w;
}
template <>
__device__ __forceinline__ void load_e<float, 2>(const float* p, float (&f)[2]) {
  const float2 v = *reinterpret_cast<const float2*>(p);
  f[0] = v.x; f[1] = v.y;
}
template <>
__device__ __forceinline__ void load_e<__nv_bfloat16, 4>(const __nv_bfloat16* p, float (&f)[4]) {
  const uint2 v = *reinterpret_cast<const uint2*>(p);
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v.y));
  f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
}
template <>
__device__ __forceinline__ void load_e<__nv_bfloat16, 2>(const __nv_bfloat16* p, float (&f)[2]) {
  const uint32_t v = *reinterpret_cast<const uint32_t*>(p);
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v));
  f[0] = a.x; f[1] = a.y;
}
template <>
__device__ __forceinline__ void load_e<__half, 4>(const __half* p, float (&f)[4]) {
  const uint2 v = *reinterpret_cast<const uint2*>(p);
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&v.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&v.y));
  f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
}
template <>
__device__ __forceinline__ void load_e<__half, 2>(const __half* p, float (&f)[2]) {
  const uint32_t v = *reinterpret_cast<const uint32_t*>(p);
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&v));
  f[0] = a.x; f[1] = a.y;
}

template <typename T>
__device__ __forceinline__ T to_t(float v);
template <>
__device__ __forceinline__ float to_t<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half to_t<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 to_t<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

constexpr int kGqaWarps = 4;
constexpr int kUnroll = 8;  // K/V rows per warp in flight (x2 for K and V)

template <typename T, int D, int GMAX>
__global__ void __launch_bounds__(32 * kGqaWarps)
    gqa_decode_split_kernel(const GqaParams p) {
  constexpr int E = D / 32;  // elements of a row per lane
  __shared__ float sm_m[kGqaWarps][GMAX];
  __shared__ float sm_l[kGqaWarps][GMAX];
  __shared__ float sm_acc[kGqaWarps][GMAX][D];

  const int kvh = blockIdx.x, b = blockIdx.y, split = blockIdx.z;
  const int warp = static_cast<int>(threadIdx.x >> 5), lane = static_cast<int>(threadIdx.x & 31);
  const int G = p.G;
  const int t_begin = split * p.tokens_per_split;
  const int t_end = min(p.T, t_begin + p.tokens_per_split);

  const T* qp = static_cast<const T*>(p.q) + (static_cast<int64_t>(b) * p.Hq + kvh * G) * D;
  float q[GMAX][E];
#pragma unroll
  for (int g = 0; g < GMAX; ++g) {
    if (g < G) {
      load_e<T, E>(qp + g * D + lane * E, q[g]);
#pragma unroll
      for (int e = 0; e < E; ++e) q[g][e] *= p.qscale;
    } else {
#pragma unroll
      for (int e = 0; e < E; ++e) q[g][e] = 0.f;
    }
  }
  float m[GMAX], l[GMAX], acc[GMAX][E];
#pragma unroll
  for (int g = 0; g < GMAX; ++g) {
    m[g] = -FLT_MAX;
    l[g] = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) acc[g][e] = 0.f;
  }

  const int64_t tstride = static_cast<int64_t>(p.Hkv) * D;  // elements between tokens
  const int64_t base = (static_cast<int64_t>(b) * p.T * p.Hkv + kvh) * D + lane * E;
  const T* kp = static_cast<const T*>(p.k) + base;
  const T* vp = static_cast<const T*>(p.v) + base;
  // Each warp takes runs of kUnroll consecutive tokens (every kGqaWarps-th
  // run) and issues all of a run's K and V row loads before using any, so a
  // warp keeps 2 * kUnroll rows in flight instead of waiting on each.
  for (int tb = t_begin + warp * kUnroll; tb < t_end; tb += kGqaWarps * kUnroll) {
    float kf[kUnroll][E], vf[kUnroll][E];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int t = tb + u < t_end ? tb + u : tb;  // clamp: the load stays in bounds
      load_e<T, E>(kp + t * tstride, kf[u]);
      load_e<T, E>(vp + t * tstride, vf[u]);
    }
    // All scores of the run first: kUnroll * G independent shuffle-reduction
    // chains that interleave, instead of one dependent chain per token.
    float sc[kUnroll][GMAX];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u)
#pragma unroll
      for (int g = 0; g < GMAX; ++g) {
        float d = 0.f;
#pragma unroll
        for (int e = 0; e < E; ++e) d = fmaf(q[g][e], kf[u][e], d);
        sc[u][g] = d;
      }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int u = 0; u < kUnroll; ++u)
#pragma unroll
        for (int g = 0; g < GMAX; ++g)
          if (g < G) sc[u][g] += __shfl_xor_sync(0xffffffffu, sc[u][g], o);
    // One online-softmax rescale per run and head.
#pragma unroll
    for (int g = 0; g < GMAX; ++g) {
      if (g >= G) continue;
      float mx = m[g];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u)
        if (tb + u < t_end) mx = fmaxf(mx, sc[u][g]);
      const float c = exp2f(m[g] - mx);
      l[g] *= c;
#pragma unroll
      for (int e = 0; e < E; ++e) acc[g][e] *= c;
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        if (tb + u < t_end) {
          const float pw = exp2f(sc[u][g] - mx);
          l[g] += pw;
#pragma unroll
          for (int e = 0; e < E; ++e) acc[g][e] = fmaf(pw, vf[u][e], acc[g][e]);
        }
      }
      m[g] = mx;
    }
  }
#pragma unroll
  for (int g = 0; g < GMAX; ++g) {
    if (g < G) {
#pragma unroll
      for (int e = 0; e < E; ++e) sm_acc[warp][g][lane * E + e] = acc[g][e];
      if (lane == 0) {
        sm_m[warp][g] = m[g];
        sm_l[warp][g] = l[g];
      }
    }
  }
  __syncthreads();

  const int h0 = kvh * G;
  for (int idx = static_cast<int>(threadIdx.x); idx < G * D; idx += 32 * kGqaWarps) {
    const int g = idx / D, d = idx % D;
    float mx = -FLT_MAX;
#pragma unroll
    for (int w = 0; w < kGqaWarps; ++w) mx = fmaxf(mx, sm_m[w][g]);
    float num = 0.f, den = 0.f;
#pragma unroll
    for (int w = 0; w < kGqaWarps; ++w) {
      const float f = exp2f(sm_m[w][g] - mx);
      num = fmaf(sm_acc[w][g][d], f, num);
      den = fmaf(sm_l[w][g], f, den);
    }
    const int64_t row = static_cast<int64_t>(b) * p.Hq + h0 + g;  // (batch, q head)
    if (p.S == 1) {
      static_cast<T*>(p.out)[row * D + d] = to_t<T>(num / den);
    } else {
      const int64_t slot = row * p.S + split;
      p.ws_acc[slot * D + d] = num;
      if (d == 0) {
        p.ws_ml[slot * 2] = mx;
        p.ws_ml[slot * 2 + 1] = den;
      }
    }
  }
}

// Merge of the S split partials of one (batch, head): out = sum_s acc_s *
// 2^(m_s - M) / sum_s l_s * 2^(m_s - M), M = max_s m_s.
template <typename T>
__global__ void gqa_decode_merge_kernel(const GqaParams p, int D) {
  const int64_t row = blockIdx.x;
  const float* ml = p.ws_ml + row * p.S * 2;
  float mx = -FLT_MAX;
  for (int s = 0; s < p.S; ++s) mx = fmaxf(mx, ml[s * 2]);
  for (int d = static_cast<int>(threadIdx.x); d < D; d += blockDim.x) {
    float num = 0.f, den = 0.f;
    for (int s = 0; s < p.S; ++s) {
      const float f = exp2f(ml[s * 2] - mx);
      num = fmaf(p.ws_acc[(row * p.S + s) * D + d], f, num);
      den = fmaf(ml[s * 2 + 1], f, den);
    }
    static_cast<T*>(p.out)[row * D + d] = to_t<T>(num / den);
  }
}

// Context splits per (batch, KV head): as many as keep every CTA resident in
// one wave (three per SM), at least 32 tokens per split, and no more than the
// workspace holds.
int gqa_choose_splits(int64_t B, int64_t Hq, int64_t Hkv, int64_t D, int64_t T, int sms,
                      size_t workspace_bytes) {
  // All CTAs resident at once: three per SM fit (registers), and a second
  // partial wave would double the time.
  const int64_t ctas = B * Hkv;
  int64_t s = (3 * static_cast<int64_t>(sms)) / (ctas > 0 ? ctas : 1);
  const int64_t by_len = (T + 31) / 32;
  if (s > by_len) s = by_len;
  if (s > 64) s = 64;
  if (s < 1) s = 1;
  while (s > 1 && gqa_workspace_bytes(B, Hq, D, s) > workspace_bytes) --s;
  return static_cast<int>(s);
}

size_t gqa_workspace_bytes(int64_t B, int64_t Hq, int64_t D, int64_t S) {
  if (S <= 1) return 0;
  return static_cast<size_t>(B * Hq * S) * static_cast<size_t>(D + 2) * sizeof(float);
}

// CTAs of this instantiation that fit on one SM (registers decide).
template <typename T, int D, int GMAX>
static int gqa_blocks_per_sm() {
  static int cache[kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev >= kMaxDevices) return 1;
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, gqa_decode_split_kernel<T, D, GMAX>,
                                                      32 * kGqaWarps, 0) != cudaSuccess ||
        n < 1) {
      cudaGetLastError();
      n = 1;
    }
    cache[dev] = n;
  }
  return cache[dev];
}

template <typename T, int D>
static int launch_gqa_t(const GqaProblem& g, int S, cudaStream_t stream) {
  {  // keep every CTA resident: no second partial wave
    int dev = 0;
    cudaGetDevice(&dev);
    const int bps = g.Hq / g.Hkv <= 4 ? gqa_blocks_per_sm<T, D, 4>() : gqa_blocks_per_sm<T, D, 8>();
    const int64_t fit = static_cast<int64_t>(bps) * sm_count(dev) / (g.B * g.Hkv);
    if (S > fit) S = fit > 1 ? static_cast<int>(fit) : 1;
  }
  GqaParams p;
  p.q = g.q;
  p.k = g.k;
  p.v = g.v;
  p.out = g.out;
  p.B = static_cast<int32_t>(g.B);
  p.Hq = static_cast<int32_t>(g.Hq);
  p.Hkv = static_cast<int32_t>(g.Hkv);
  p.T = static_cast<int32_t>(g.T);
  p.G = static_cast<int32_t>(g.Hq / g.Hkv);
  p.S = S;
  p.tokens_per_split = static_cast<int32_t>((g.T + S - 1) / S);
  p.qscale = g.scale * 1.4426950408889634f;  // log2(e): the softmax runs in base 2
  float* ws = static_cast<float*>(g.workspace);
  p.ws_acc = S > 1 ? ws : nullptr;
  p.ws_ml = S > 1 ? ws + static_cast<int64_t>(g.B) * g.Hq * S * D : nullptr;
  const dim3 grid(static_cast<unsigned>(g.Hkv), static_cast<unsigned>(g.B),
                  static_cast<unsigned>(S));
  if (p.G <= 4)
    gqa_decode_split_kernel<T, D, 4><<<grid, 32 * kGqaWarps, 0, stream>>>(p);
  else
    gqa_decode_split_kernel<T, D, 8><<<grid, 32 * kGqaWarps, 0, stream>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error("launch gqa_decode_split", e);
  if (S > 1) {
    gqa_decode_merge_kernel<T><<<static_cast<unsigned>(g.B * g.Hq), D, 0, stream>>>(p, D);
    e = cudaGetLastError();
    if (e != cudaSuccess) return set_cuda_error("launch gqa_decode_merge", e);
  }
  return 0;
}

template <typename T>
static int launch_gqa_d(const GqaProblem& g, int S, cudaStream_t s) {
  if (g.D == 128) return launch_gqa_t<T, 128>(g, S, s);
  return launch_gqa_t<T, 64>(g, S, s);
}

// Device address of g_gqa_noalloc_scratch, looked up once per device with
// that device current (the caller's current device).
int gqa_noalloc_scratch(int dev, void** ptr) {
  static std::mutex mu;
  static void* cache[kMaxDevices] = {};
  if (dev < 0 || dev >= kMaxDevices)
    return set_error(FRN_ERR_UNSUPPORTED, "device %d out of range for the static scratch", dev);
  std::lock_guard<std::mutex> lock(mu);
  if (!cache[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_gqa_noalloc_scratch);
    if (e != cudaSuccess) return set_cuda_error("cudaGetSymbolAddress(GQA decode scratch)", e);
    cache[dev] = p;
  }
  *ptr = cache[dev];
  return 0;
}

size_t gqa_noalloc_scratch_bytes() { return kGqaNoAllocScratchBytes; }

int run_gqa_decode(const GqaProblem& g, int splits, cudaStream_t s) {
  if (gqa_mma_supported(g)) return run_gqa_decode_mma(g, splits, s);
  switch (g.dtype) {
    case FRN_DTYPE_BF16: return launch_gqa_d<__nv_bfloat16>(g, splits, s);
    case FRN_DTYPE_F16: return launch_gqa_d<__half>(g, splits, s);
    case FRN_DTYPE_F32: return launch_gqa_d<float>(g, splits, s);
    default: return set_error(FRN_ERR_UNSUPPORTED, "GQA decode supports fp32, fp16 and bf16");
  }
}

}  // namespace frn
