// frn_gqa_decode_mma.cu -- decode-step grouped-query attention on tensor
// cores (bf16 / fp16, head dim 64 or 128, up to 8 query heads per KV head).
//
// Same contract and split/merge structure as frn_gqa_decode.cu; the per-token
// work moves from warp shuffles to 16x8x16 MMAs.  For one (batch, KV head)
// the G query heads are the M rows of the MMA (rows G..15 are zero), so
//
//   S  = Q . K^T   M = heads, N = 8 tokens, K = 16 head dims per MMA
//   O += P . V     M = heads, N = 8 head dims, K = 16 tokens per MMA
//
// and the softmax runs on the accumulator fragments: per 16-token block a
// row max and a rescale cost two shuffles, instead of a shuffle reduction per
// token and head.  P is rounded to the input type for the second MMA (its
// fp32 row sums are kept for the normalisation).
//
// CTA (KV head, batch, split), 192 threads: warps 4 and 5 load 64-token K
// and V stages with TMA (a 3-D view (d, KV head, token) of the cache, 64-d
// boxes with the 128-byte swizzle) into a 4-slot ring; warps 0-3 each take 16
// tokens of every stage: ldmatrix (K as the B operand of S, V transposed as
// the B operand of O), MMAs, online softmax in base 2.  Tokens past the
// split's end read as -inf scores.  The four warps merge in shared memory;
// with one split the CTA writes the output, otherwise the S <= 8 splits of a
// (batch, KV head) are one thread-block cluster: CTA r owns a 1/S slice of
// the G*D outputs, every CTA pushes its (acc, max, sum) for each slice into
// the owner's receive buffer with st.shared::cluster, and after one cluster
// barrier each owner combines its slice from local shared memory in rank
// order (no workspace, no second launch, no remote loads).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cfloat>
#include <cstdint>

#include "frn_internal.h"
#include "frn_ptx.cuh"

namespace frn {

struct GqaMmaParams {
  const void* q;
  void* out;
  int32_t B, Hq, Hkv, T, G, S, tokens_per_split;
  float qscale;  // scale * log2(e)
  uint64_t timeout_ns;
};

constexpr int kGqaStageTokens = 64;
constexpr int kGqaRing = 4;

template <int D>
struct GqaMmaCfg {
  static constexpr int HALVES = D / 64;                   // 64-d boxes per row
  static constexpr int HALF_BYTES = kGqaStageTokens * 128;  // [64 tokens x 64 d]
  static constexpr int STAGE_BYTES = 2 * HALVES * HALF_BYTES;  // K then V
  static constexpr int OFF_BAR = kGqaRing * STAGE_BYTES;
  // Cluster-merge receive buffer, a space of its own (peers may write it
  // while this CTA still streams): acc [S][ceil(G*D/S)] (<= 8*D + 7 floats)
  // then max and sum [S][16].
  static constexpr int OFF_RECV = OFF_BAR + 128;
  static constexpr int RECV_ACC_FLOATS = 8 * D + 8;
  static constexpr int RECV_FLOATS = RECV_ACC_FLOATS + 8 * 16;
  static constexpr int SMEM_BYTES = OFF_RECV + RECV_FLOATS * 4 + 1024;
  static constexpr int THREADS = 192;
  // The warp merge reuses the ring: [4 warps][8 heads][D] acc + m + l.
  static constexpr int MERGE_FLOATS = 4 * 8 * D + 2 * 4 * 8;
  static_assert(MERGE_FLOATS * 4 <= OFF_BAR, "merge buffers fit in the ring");
  static_assert(2 * kGqaRing * 8 + 4 <= 128, "barriers and flag fit before the receive buffer");
};

template <typename T>
__device__ __forceinline__ void mma_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                          uint32_t b1);
template <>
__device__ __forceinline__ void mma_16816<__nv_bfloat16>(float (&c)[4], const uint32_t (&a)[4],
                                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, "
      "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma_16816<__half>(float (&c)[4], const uint32_t (&a)[4],
                                                  uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, "
      "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr)
               : "memory");
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr)
               : "memory");
}

template <typename T>
__device__ __forceinline__ T to_out(float v);
template <>
__device__ __forceinline__ __nv_bfloat16 to_out<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
template <>
__device__ __forceinline__ __half to_out<__half>(float v) {
  return __float2half_rn(v);
}

// Barrier among the four compute warps (the loader warps skip the merge).
__device__ __forceinline__ void bar_sync_compute() {
  asm volatile("bar.sync 1, 128;" ::: "memory");
}

// Byte offset of 16-byte chunk `c` (0..7) of token row `tok` in a [64 x 128 B]
// box written with the 128-byte swizzle.
__device__ __forceinline__ uint32_t sw128(int tok, int c) {
  return static_cast<uint32_t>(tok * 128 + ((c ^ (tok & 7)) << 4));
}

template <typename T, int D>
__global__ void __launch_bounds__(GqaMmaCfg<D>::THREADS, 2)
    gqa_decode_mma_kernel(const __grid_constant__ CUtensorMap tmap_k,
                          const __grid_constant__ CUtensorMap tmap_v, const GqaMmaParams p) {
  using C = GqaMmaCfg<D>;
  constexpr int NKC = D / 16;  // 16-d chunks of S's reduction
  constexpr int NDT = D / 8;   // 8-d output tiles of O
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* empty = full + kGqaRing;
  volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(empty + kGqaRing);

  const int kvh = blockIdx.x, b = blockIdx.y, split = blockIdx.z;
  const int warp = static_cast<int>(threadIdx.x >> 5), lane = static_cast<int>(threadIdx.x & 31);
  const int G = p.G;
  const int t_begin = split * p.tokens_per_split;
  const int t_end = min(p.T, t_begin + p.tokens_per_split);
  const int nstages = (t_end - t_begin + kGqaStageTokens - 1) / kGqaStageTokens;
  const uint64_t to = p.timeout_ns;

  if (threadIdx.x == 0) {
    prefetch_tmap(&tmap_k);
    prefetch_tmap(&tmap_v);
    for (int s = 0; s < kGqaRing; ++s) {
      mbar_init(&full[s], 2);   // K and V loaders, with their bytes
      mbar_init(&empty[s], 4);  // the four compute warps
    }
    *abort_flag = 0u;
    fence_mbarrier_init();
  }
  __syncthreads();
  // Peers write this CTA's receive buffer only after this rendezvous (every
  // CTA of the cluster has started).
  if (p.S > 1) {
    cluster_arrive_relaxed();
    cluster_wait();
  }
  // The next grid in the stream may start its set-up now; everything this
  // grid reads or writes in global memory waits for the previous grid.
  griddep_launch_dependents();
  griddep_wait();

  if (warp >= 4) {
    // Loader: warp 4 streams K, warp 5 streams V (HALVES boxes per stage).
    // It takes part in the cluster barriers at the end, nothing else.
    if (lane == 0) {
      const bool is_v = warp == 5;
      const CUtensorMap* m = is_v ? &tmap_v : &tmap_k;
      const int row0 = b * p.T + t_begin;  // token coordinate of the split's start
      for (int i = 0; i < nstages; ++i) {
        const int s = i % kGqaRing;
        const uint32_t ph = static_cast<uint32_t>(i / kGqaRing) & 1u;
        if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, to)) {
          __nanosleep(20000);  // loads already issued may still be landing
          break;
        }
        mbar_arrive_expect_tx(&full[s], C::HALVES * C::HALF_BYTES);
        uint8_t* dst = smem + s * C::STAGE_BYTES + (is_v ? C::HALVES * C::HALF_BYTES : 0);
#pragma unroll
        for (int h = 0; h < C::HALVES; ++h)
          tma_load_3d(dst + h * C::HALF_BYTES, m, &full[s], h * 64, kvh,
                      row0 + i * kGqaStageTokens);
      }
    }
  } else {
  // ---- compute warps: fragment coordinates
  const int g = lane >> 2, tq = lane & 3;
  // Q as the A operand of S: rows = heads (g < G real), k = head dims.
  uint32_t qa[NKC][2];  // a0 (row g, d 16kc+2tq..+1), a2 (row g, d 16kc+8+2tq..+1)
  {
    const T* qp = static_cast<const T*>(p.q) + (static_cast<int64_t>(b) * p.Hq + kvh * G + g) * D;
#pragma unroll
    for (int kc = 0; kc < NKC; ++kc) {
      qa[kc][0] = g < G ? *reinterpret_cast<const uint32_t*>(qp + kc * 16 + 2 * tq) : 0u;
      qa[kc][1] = g < G ? *reinterpret_cast<const uint32_t*>(qp + kc * 16 + 8 + 2 * tq) : 0u;
    }
  }
  float o[NDT][4];
#pragma unroll
  for (int j = 0; j < NDT; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_run = -FLT_MAX;  // row g's running max (base 2); rows g+8 are padding
  float l_run = 0.f;       // this thread's part of row g's sum

  const uint32_t ring = smem_addr(smem);
  // ldmatrix row addresses: thread i feeds row (i & 7) of matrix (i >> 3).
  const int mi = lane >> 3, mr = lane & 7;
  // K (non-transposed): matrices (tok 0-7 | 8-15) x (d lo | hi 8 of a 16-d chunk)
  const int k_tok = warp * 16 + ((mi >> 1) << 3) + mr;
  const int k_hi = mi & 1;
  // V (transposed): matrices (tok 0-7 | 8-15) x (d tile j | j+1)
  const int v_tok = warp * 16 + ((mi & 1) << 3) + mr;
  const int v_next = mi >> 1;

  for (int i = 0; i < nstages; ++i) {
    const int s = i % kGqaRing;
    const uint32_t ph = static_cast<uint32_t>(i / kGqaRing) & 1u;
    if (!mbar_wait(&full[s], ph, abort_flag, to)) break;
    const uint32_t kbase = ring + s * C::STAGE_BYTES;
    const uint32_t vbase = kbase + C::HALVES * C::HALF_BYTES;

    // S = Q . K^T for this warp's 16 tokens: two 8-token tiles.
    float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int kc = 0; kc < NKC; ++kc) {
      const int h = kc / 4;                       // 64-d box
      const int c = (kc % 4) * 2 + k_hi;          // 16-byte chunk within the row
      uint32_t kb[4];
      ldsm_x4(kbase + h * C::HALF_BYTES + sw128(k_tok, c), kb);
      const uint32_t a[4] = {qa[kc][0], 0u, qa[kc][1], 0u};
      mma_16816<T>(sc[0], a, kb[0], kb[1]);
      mma_16816<T>(sc[1], a, kb[2], kb[3]);
    }
    // Online softmax on row g (columns: tokens 2tq, 2tq+1 of each tile).
    const int tok0 = t_begin + i * kGqaStageTokens + warp * 16 + 2 * tq;
    float x[4];
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int tok = tok0 + n * 8 + e;
        x[n * 2 + e] = tok < t_end ? sc[n][e] * p.qscale : -INFINITY;
      }
    float bm = fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3]));
    bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 1));
    bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 2));
    const float m_new = fmaxf(m_run, bm);
    const float corr = exp2f(m_run - m_new);
    m_run = m_new;
    float pr[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) pr[e] = exp2f(x[e] - m_new);
    l_run = l_run * corr + (pr[0] + pr[1]) + (pr[2] + pr[3]);
#pragma unroll
    for (int j = 0; j < NDT; ++j) {
      o[j][0] *= corr;
      o[j][1] *= corr;
    }
    // P as the A operand of O += P . V (k = the 16 tokens): rows g+8 are zero.
    const uint32_t pa[4] = {float2_to_pair<T>(pr[0], pr[1]), 0u, float2_to_pair<T>(pr[2], pr[3]),
                            0u};
#pragma unroll
    for (int j = 0; j < NDT; j += 2) {
      const int d0 = (j + v_next) * 8;
      uint32_t vb[4];
      ldsm_x4_trans(vbase + (d0 / 64) * C::HALF_BYTES + sw128(v_tok, (d0 % 64) / 8), vb);
      mma_16816<T>(o[j], pa, vb[0], vb[1]);
      mma_16816<T>(o[j + 1], pa, vb[2], vb[3]);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }

  if (*abort_flag) __nanosleep(20000);  // a wait ran out: let issued loads land
  // Row sums over the four threads of each row.
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);

  // Merge the four warps (the ring is free once every warp is past its loop).
  bar_sync_compute();
  float* sm_acc = reinterpret_cast<float*>(smem);  // [4][8][D]
  float* sm_m = sm_acc + 4 * 8 * D;                // [4][8]
  float* sm_l = sm_m + 4 * 8;                      // [4][8]
  if (g < G) {
#pragma unroll
    for (int j = 0; j < NDT; ++j) {
      sm_acc[(warp * 8 + g) * D + j * 8 + 2 * tq] = o[j][0];
      sm_acc[(warp * 8 + g) * D + j * 8 + 2 * tq + 1] = o[j][1];
    }
    if (tq == 0) {
      sm_m[warp * 8 + g] = m_run;
      sm_l[warp * 8 + g] = l_run;
    }
  }
  bar_sync_compute();
  const int h0 = kvh * G;
  for (int idx = static_cast<int>(threadIdx.x); idx < G * D; idx += 128) {
    const int gg = idx / D, d = idx % D;
    float mx = -FLT_MAX;
#pragma unroll
    for (int w = 0; w < 4; ++w) mx = fmaxf(mx, sm_m[w * 8 + gg]);
    float num = 0.f, den = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float f = exp2f(sm_m[w * 8 + gg] - mx);
      num = fmaf(sm_acc[(w * 8 + gg) * D + d], f, num);
      den = fmaf(sm_l[w * 8 + gg], f, den);
    }
    const int64_t row = static_cast<int64_t>(b) * p.Hq + h0 + gg;
    if (p.S == 1) {
      static_cast<T*>(p.out)[row * D + d] = to_out<T>(num / den);
    } else {
      // Output idx belongs to CTA idx / chunk; this CTA's (split's) values go
      // to slot [split][idx % chunk] of its receive buffer, and every owner
      // gets this CTA's max and sum of head gg.
      const int chunk = (G * D + p.S - 1) / p.S;
      const uint32_t recv_a = smem_addr(smem + C::OFF_RECV);
      const int owner = idx / chunk;
      st_shared_cluster_f32(
          mapa_shared(recv_a + static_cast<uint32_t>(split * chunk + idx - owner * chunk) * 4u,
                      static_cast<uint32_t>(owner)),
          num);
      if (d == 0) {
        const uint32_t ml_a = recv_a + (C::RECV_ACC_FLOATS + split * 16 + gg) * 4;
        for (int r = 0; r < p.S; ++r) {
          st_shared_cluster_f32(mapa_shared(ml_a, static_cast<uint32_t>(r)), mx);
          st_shared_cluster_f32(mapa_shared(ml_a + 8 * 4, static_cast<uint32_t>(r)), den);
        }
      }
    }
  }
  }  // compute warps

  if (p.S > 1) {
    // Cluster merge: CTA `split` (its rank) combines outputs [lo, hi) of the
    // G*D from all S CTAs, in rank order, out of its own receive buffer.
    // After this barrier no CTA touches a peer's shared memory, so none
    // waits for the others before leaving.
    cluster_sync_all();
    if (warp < 4 && !*abort_flag) {
      const float* racc = reinterpret_cast<const float*>(smem + C::OFF_RECV);
      const float* rml = racc + C::RECV_ACC_FLOATS;  // [S][16]: max [8], sum [8]
      const int total = G * D, chunk = (total + p.S - 1) / p.S;
      const int lo = split * chunk, hi = min(total, lo + chunk);
      for (int idx = lo + static_cast<int>(threadIdx.x); idx < hi; idx += 128) {
        const int gg = idx / D, d = idx % D;
        float ms[8], mx = -FLT_MAX;
        for (int r = 0; r < p.S; ++r) {
          ms[r] = rml[r * 16 + gg];
          mx = fmaxf(mx, ms[r]);
        }
        float num = 0.f, den = 0.f;
        for (int r = 0; r < p.S; ++r) {
          const float f = exp2f(ms[r] - mx);
          num = fmaf(racc[r * chunk + idx - lo], f, num);
          den = fmaf(rml[r * 16 + 8 + gg], f, den);
        }
        const int64_t row = static_cast<int64_t>(b) * p.Hq + kvh * G + gg;
        static_cast<T*>(p.out)[row * D + d] = to_out<T>(num / den);
      }
    }
  }
}

// ------------------------------------------------------------------ host side

template <typename T, int D>
static int launch_gqa_mma(const GqaProblem& g, int S, cudaStream_t stream) {
  using C = GqaMmaCfg<D>;
  auto kern = gqa_decode_mma_kernel<T, D>;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return set_cuda_error("cudaGetDevice");
  static int bps[kMaxDevices] = {};
  if (dev < kMaxDevices && bps[dev] == 0) {
    cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
    if (e != cudaSuccess) return set_cuda_error("cudaFuncSetAttribute(gqa mma kernel)", e);
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, C::THREADS, C::SMEM_BYTES) !=
            cudaSuccess ||
        n < 1) {
      cudaGetLastError();
      n = 1;
    }
    bps[dev] = n;
  }
  // Every CTA resident in one wave, and at least one 64-token stage a split.
  const int64_t fit = static_cast<int64_t>(dev < kMaxDevices ? bps[dev] : 1) * sm_count(dev) /
                      (g.B * g.Hkv);
  if (S > fit) S = fit > 1 ? static_cast<int>(fit) : 1;
  const int64_t by_len = (g.T + kGqaStageTokens - 1) / kGqaStageTokens;
  if (S > by_len) S = static_cast<int>(by_len);
  if (S > 8) S = 8;  // the splits of a (batch, KV head) form one portable cluster
  if (S < 1) S = 1;

  const CUtensorMapDataType dt = Elem16<T>::kTmaType;
  // (d, KV head, token) view of [B*T, Hkv, D]: 64-d boxes of 64 tokens.
  const uint64_t dims[3] = {static_cast<uint64_t>(D), static_cast<uint64_t>(g.Hkv),
                            static_cast<uint64_t>(g.B * g.T)};
  const uint64_t strides[2] = {static_cast<uint64_t>(D) * 2,
                               static_cast<uint64_t>(g.Hkv) * D * 2};
  const uint32_t box[3] = {64, 1, kGqaStageTokens};
  CUtensorMap tk, tv;
  int rc = encode_tmap_3d(&tk, dt, g.k, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = encode_tmap_3d(&tv, dt, g.v, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;

  GqaMmaParams p;
  p.q = g.q;
  p.out = g.out;
  p.B = static_cast<int32_t>(g.B);
  p.Hq = static_cast<int32_t>(g.Hq);
  p.Hkv = static_cast<int32_t>(g.Hkv);
  p.T = static_cast<int32_t>(g.T);
  p.G = static_cast<int32_t>(g.Hq / g.Hkv);
  p.S = S;
  p.tokens_per_split = static_cast<int32_t>((g.T + S - 1) / S);
  p.qscale = g.scale * 1.4426950408889634f;  // log2(e): the softmax runs in base 2
  p.timeout_ns = wait_timeout_ns();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(g.Hkv), static_cast<unsigned>(g.B),
                     static_cast<unsigned>(S));
  cfg.blockDim = dim3(C::THREADS);
  cfg.dynamicSmemBytes = C::SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[2];
  attrs[0].id = cudaLaunchAttributeClusterDimension;
  attrs[0].val.clusterDim.x = 1;
  attrs[0].val.clusterDim.y = 1;
  attrs[0].val.clusterDim.z = static_cast<unsigned>(S);
  attrs[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attrs;
  cfg.numAttrs = 2;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, tk, tv, p);
  if (e != cudaSuccess) return set_cuda_error("launch gqa_decode_mma", e);
  return 0;
}

bool gqa_mma_supported(const GqaProblem& g) {
  const int64_t G = g.Hkv > 0 ? g.Hq / g.Hkv : 0;
  return (g.dtype == FRN_DTYPE_BF16 || g.dtype == FRN_DTYPE_F16) && (g.D == 64 || g.D == 128) &&
         G >= 1 && G <= 8 && g.T >= 1;
}

int run_gqa_decode_mma(const GqaProblem& g, int splits, cudaStream_t s) {
  if (g.dtype == FRN_DTYPE_BF16)
    return g.D == 128 ? launch_gqa_mma<__nv_bfloat16, 128>(g, splits, s)
                      : launch_gqa_mma<__nv_bfloat16, 64>(g, splits, s);
  return g.D == 128 ? launch_gqa_mma<__half, 128>(g, splits, s)
                    : launch_gqa_mma<__half, 64>(g, splits, s);
}

}  // namespace frn
