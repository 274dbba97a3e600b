// frn_decode.cu -- fused RMSNorm -> Linear for decode batches (M <= 128).
//
// With few tokens the op is a weight stream: W [N, K] dominates the bytes
// (Llama-3-8B QKV: 50 MB of W against 8 KB - 1 MB of x), so the kernel is
// built to keep ~all SMs pulling W from HBM:
//
//   swap-AB   D^T[n, t] = W[n, :] . x[t, :]: a 128-row W tile is the UMMA M
//             operand, the MP (16/32/64/128) padded tokens are UMMA N, the
//             fp32 accumulator sits in TMEM (lane = W row, column = token).
//   split-K   the CTAs of one thread-block cluster (S <= 8) share a W tile and
//             each streams 1/S of K, so N/128 * S CTAs cover the SMs.
//   reduce    each CTA writes its fp32 partial D^T and its partial sum of x^2
//             per token into its own shared memory; after a cluster barrier,
//             CTA r reduces tokens t = r, r+S, ... by reading the S partials
//             through distributed shared memory in rank order (deterministic,
//             no atomics, no global workspace), applies
//             inv_rms[t] = rsqrt(sum_s ss_s[t] / K + eps) and b[n], and stores
//             out[t, n0 .. n0+127] as coalesced rows.
//
// SwiGLU variant: a tile is 64 gate rows over the matching 64 up rows, and
// the reduction combines the two halves into 64 output columns.
//
// Roles: warps 0-3 epilogue (TMEM lanes -> partial buffer) and reduction,
// warps 4-7 TMA producers (W / x over even / odd stages), warps 8 and 13 MMA
// issuers of the even / odd k-blocks into two accumulators (warp 8 also owns
// TMEM), warps 9-12 RMS (thread t sums x[t, k-range]^2 from x stages).
//
// Two issuers: a chain of MMAs into one accumulator completes one 128 x MP x
// 16 MMA only every ~115-190 clocks however small MP is, so with one chain
// the MMAs fell behind the weight stream and finished ~2 us after the last
// k-block arrived; two independent chains (summed in the epilogue) keep up.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "frn_internal.h"
#include "frn_ptx.cuh"

namespace frn {

struct DecodeParams {
  int32_t M, N, K;
  int32_t num_k_blocks;
  int32_t split;  // CTAs per cluster (k-splits)
  float eps;
  const void* bias;
  // Output parts: columns [part_col0[i], part_col0[i+1]) go to part_out[i]
  // (row stride part_stride[i]); one part is the plain [M, N] output.
  int32_t nparts;
  int32_t part_col0[kMaxParts];
  void* part_out[kMaxParts];
  int64_t part_stride[kMaxParts];
  int32_t up_row0;  // SwiGLU: first W row of the up block (= intermediate)
  uint64_t timeout_ns;
};

__device__ __forceinline__ float ld_shared_cluster_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

__device__ __forceinline__ float2 ld_shared_cluster_f32x2(uint32_t addr) {
  float2 v;
  asm volatile("ld.shared::cluster.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(addr)
               : "memory");
  return v;
}

template <int MP, int STAGES>
struct DecodeCfg {
  static constexpr int BM = 128;  // W rows per tile
  static constexpr int BK = 64;
  static constexpr int W_BYTES = BM * BK * 2;
  static constexpr int X_BYTES = MP * BK * 2;
  static constexpr int STAGE_TX = W_BYTES + X_BYTES;
  static constexpr uint32_t TMEM_COLS = 2 * MP < 32 ? 32u : static_cast<uint32_t>(2 * MP);
  static constexpr int OFF_W = 0;
  static constexpr int OFF_X = OFF_W + STAGES * W_BYTES;
  static constexpr int PART_BYTES = MP * BM * 4;  // fp32 partial D, [token][w row]
  static constexpr int PIPE_BYTES = STAGES * (W_BYTES + X_BYTES);
  static constexpr int OFF_SS = (PIPE_BYTES > PART_BYTES ? PIPE_BYTES : PART_BYTES);
  static constexpr int OFF_BAR = OFF_SS + 128 * 4;
  static constexpr int NUM_BARS = 2 * STAGES + 3;
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
  static constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;
  // warps 4-7: producers (W | x) x (even | odd stages); 8, 13: MMA; 9-12: RMS
  static constexpr int WARP_PROD0 = 4, WARP_MMA = 8, WARP_RMS0 = 9, WARP_MMA1 = 13;
  static constexpr int THREADS = 32 * 14;
  static_assert(STAGES % 2 == 0, "stages alternate between two producers and two issuers");
  static_assert(MP % 16 == 0 && MP >= 16 && MP <= 128, "MP");
  static_assert(X_BYTES % 1024 == 0, "x stages must stay 1024-aligned");
  // The partial buffer may only overlap the W stages (read by the MMA alone),
  // never the x stages, which RMS warps can still be reading.
  static_assert(PART_BYTES <= STAGES * W_BYTES, "partial buffer overlaps the x stages");
  static_assert(SMEM_BYTES <= 232448, "exceeds 227 KB of dynamic shared memory");
};

// SWIGLU: a W tile is 64 gate rows [g0, g0+64) over 64 up rows [I+g0, ...)
// (two TMA boxes of 64 rows), and the reduction writes output columns
// g0 + c = silu(D[c] * inv_rms + b[g0+c]) * (D[64+c] * inv_rms + b[I+g0+c]).
template <typename T, int MP, int STAGES, bool SWIGLU>
__global__ void __launch_bounds__(DecodeCfg<MP, STAGES>::THREADS, 1)
    fused_rmsnorm_linear_decode_kernel(const __grid_constant__ CUtensorMap tmap_w,
                                       const __grid_constant__ CUtensorMap tmap_x,
                                       const DecodeParams p) {
  using C = DecodeCfg<MP, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* empty = full + STAGES;
  uint64_t* tmem_full = empty + STAGES;
  uint64_t* drain = tmem_full + 1;  // [issuer]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile uint32_t* abort_flag = tmem_slot + 1;
  float* part = reinterpret_cast<float*>(smem);  // reuses the pipeline buffers
  float* ssq = reinterpret_cast<float*>(smem + C::OFF_SS);

  const uint32_t warp = warp_id_in_cta();
  const uint32_t lane = threadIdx.x & 31u;
  const int S = p.split;
  const uint32_t rank = cluster_cta_rank();
  const int tile = static_cast<int>(blockIdx.x) / S;
  const int n0 = tile * (SWIGLU ? C::BM / 2 : C::BM);  // first output column of the tile
  // k-blocks [kb_begin, kb_end) of this split (first splits take the remainder)
  const int base = p.num_k_blocks / S, rem = p.num_k_blocks % S;
  const int kb_begin = static_cast<int>(rank) * base + (static_cast<int>(rank) < rem ? rank : rem);
  const int nkb = base + (static_cast<int>(rank) < rem ? 1 : 0);
  const uint64_t to = p.timeout_ns;

  if (warp == C::WARP_PROD0 && lane == 0) {
    prefetch_tmap(&tmap_w);
    prefetch_tmap(&tmap_x);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 2);       // W producer + x producer arrive with tx
      mbar_init(&empty[s], 1 + 4);  // MMA commit + 4 RMS warps
    }
    mbar_init(tmem_full, 2);  // one commit per issuer
    mbar_init(&drain[0], 1);
    mbar_init(&drain[1], 1);
    *abort_flag = 0u;
    fence_mbarrier_init();
  }
  if (warp == C::WARP_MMA) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Let the next kernel in the stream get scheduled now: its CTAs take SMs as
  // ours retire and run their set-up while we finish; its griddepcontrol.wait
  // still orders all of its global accesses after this whole grid.
  griddep_launch_dependents();

  if (warp >= C::WARP_PROD0 && warp < C::WARP_PROD0 + 4) {
    // Four issuing threads (a single thread keeps only a few bulk-tensor
    // loads in flight): W / x, each over even / odd stages.
    if (lane == 0) {
      const uint32_t pid = warp - C::WARP_PROD0;
      const bool is_w = (pid & 1u) == 0;
      const uint32_t parity_sel = pid >> 1;
      // Warm L2 with this thread's first ring of tiles while the preceding
      // grid drains (see tma_prefetch_2d).
      for (int i = static_cast<int>(parity_sel); i < nkb && i < STAGES; i += 2) {
        const int kc = (kb_begin + i) * C::BK;
        if (!is_w) {
          tma_prefetch_2d(&tmap_x, kc, 0);
        } else if (SWIGLU) {
          tma_prefetch_2d(&tmap_w, kc, n0);
          tma_prefetch_2d(&tmap_w, kc, p.up_row0 + n0);
        } else {
          tma_prefetch_2d(&tmap_w, kc, n0);
        }
      }
      griddep_wait();
      uint32_t stage = 0, phase = 0;
      for (int i = 0; i < nkb; ++i) {
        if ((stage & 1u) != parity_sel) {
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
          continue;
        }
        if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, to)) break;
        const int kc = (kb_begin + i) * C::BK;
        if (is_w) {
          mbar_arrive_expect_tx(&full[stage], C::W_BYTES);
          uint8_t* wdst = smem + C::OFF_W + stage * C::W_BYTES;
          if (SWIGLU) {
            tma_load_2d(wdst, &tmap_w, &full[stage], kc, n0);
            tma_load_2d(wdst + C::W_BYTES / 2, &tmap_w, &full[stage], kc, p.up_row0 + n0);
          } else {
            tma_load_2d(wdst, &tmap_w, &full[stage], kc, n0);
          }
        } else {
          mbar_arrive_expect_tx(&full[stage], C::X_BYTES);
          tma_load_2d(smem + C::OFF_X + stage * C::X_BYTES, &tmap_x, &full[stage], kc, 0);
        }
        if (++stage == STAGES) { stage = 0; phase ^= 1u; }
      }
    }
  } else if (warp == C::WARP_MMA || warp == C::WARP_MMA1) {
    // Issuer pp: k-blocks pp, pp + 2, ... (stages of parity pp) into
    // accumulator pp at TMEM column pp * MP.
    const int pp = warp == C::WARP_MMA ? 0 : 1;
    if (lane == 0) {
      const uint32_t idesc = make_idesc_f16(Elem16<T>::kUmmaFormat, C::BM, MP);
      const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(pp * MP);
      bool ok = true;
      for (int i = pp; i < nkb; i += 2) {
        const int stage = i % STAGES;
        const uint32_t phase = static_cast<uint32_t>(i / STAGES) & 1u;
        if (!mbar_wait(&full[stage], phase, abort_flag, to)) { ok = false; break; }
        tc_fence_after();
        const uint32_t w_addr = smem_addr(smem + C::OFF_W + stage * C::W_BYTES);
        const uint32_t x_addr = smem_addr(smem + C::OFF_X + stage * C::X_BYTES);
#pragma unroll
        for (int k = 0; k < C::BK / 16; ++k)
          umma_f16_ss(d_tmem, make_smem_desc_k_sw128(w_addr + k * 32),
                      make_smem_desc_k_sw128(x_addr + k * 32), idesc, (i > pp || k > 0) ? 1u : 0u);
        umma_commit(&empty[stage]);
      }
      if (ok) umma_commit(tmem_full);
      umma_commit(&drain[pp]);
      uint32_t zero = 0;
      mbar_wait(&drain[pp], 0, &zero, to);
    }
  } else if (warp >= C::WARP_RMS0) {
    // Thread t sums x[t, k-range]^2 straight from the x stages.
    const int t = static_cast<int>(threadIdx.x) - C::WARP_RMS0 * 32;
    uint32_t stage = 0, phase = 0;
    float ss0 = 0.f, ss1 = 0.f;
    for (int i = 0; i < nkb; ++i) {
      if (!mbar_wait(&full[stage], phase, abort_flag, to)) break;
      if (t < MP) {
        const uint32_t row = smem_addr(smem + C::OFF_X + stage * C::X_BYTES) + t * 128;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const uint4 v = ld_shared_v4(row + ((q ^ (t & 7)) << 4));
          const float2 f0 = pair_to_float2<T>(v.x), f1 = pair_to_float2<T>(v.y);
          const float2 f2 = pair_to_float2<T>(v.z), f3 = pair_to_float2<T>(v.w);
          ss0 = fmaf(f0.x, f0.x, ss0); ss1 = fmaf(f0.y, f0.y, ss1);
          ss0 = fmaf(f1.x, f1.x, ss0); ss1 = fmaf(f1.y, f1.y, ss1);
          ss0 = fmaf(f2.x, f2.x, ss0); ss1 = fmaf(f2.y, f2.y, ss1);
          ss0 = fmaf(f3.x, f3.x, ss0); ss1 = fmaf(f3.y, f3.y, ss1);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[stage]);
      if (++stage == STAGES) { stage = 0; phase ^= 1u; }
    }
    // Published after the cluster barrier below, once the pipeline is idle.
    if (t < MP) ssq[t] = ss0 + ss1;
  } else {
    // Epilogue warps 0-3: accumulator lanes -> partial buffer [token][w row].
    // The pipeline buffers are reused, so wait until every MMA is done.
    const uint32_t q = warp;
    if (mbar_wait(tmem_full, 0, abort_flag, to)) {
      tc_fence_after();
      const uint32_t taddr = tmem_base + ((q * 32u) << 16);
      const int wrow = static_cast<int>(q * 32 + lane);
      const bool two = nkb >= 2;  // the odd issuer had k-blocks to accumulate
#pragma unroll 1
      for (int c = 0; c < MP / 16; ++c) {
        uint32_t v[16], v1[16];
        tmem_ld_32x32b_x16(taddr + c * 16, v);
        if (two) tmem_ld_32x32b_x16(taddr + MP + c * 16, v1);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 16; ++e)
          part[(c * 16 + e) * C::BM + wrow] =
              __uint_as_float(v[e]) + (two ? __uint_as_float(v1[e]) : 0.f);
      }
    }
  }

  // All partials (and x^2 sums) of the cluster are in shared memory.
  __syncwarp();
  tc_fence_before();
  cluster_sync_all();

  if (warp < 4 && !*abort_flag) {
    // CTA `rank` reduces tokens rank, rank+S, ...: TPT threads per token, each
    // owning output columns pr, pr+1 of the tile (W rows pr, pr+1, and for
    // SwiGLU also the up rows 64+pr, 65+pr); 128 / TPT tokens in flight.
    griddep_wait();
    constexpr int TPT = SWIGLU ? 32 : 64;
    constexpr int LANES = 128 / TPT;
    const int pr = static_cast<int>(threadIdx.x % TPT) * 2;
    const int tsub = static_cast<int>(threadIdx.x / TPT);
    const bool col_ok = n0 + pr < p.N;
    int pi = 0;  // output part of columns n0 + pr, n0 + pr + 1 (parts are 8-column multiples)
    while (pi + 1 < p.nparts && n0 + pr >= p.part_col0[pi + 1]) ++pi;
    T* const obase = static_cast<T*>(p.part_out[pi]) + (n0 + pr - p.part_col0[pi]);
    const int64_t ostride = p.part_stride[pi];
    const bool has_bias = p.bias != nullptr;
    float b0 = 0.f, b1 = 0.f, bu0 = 0.f, bu1 = 0.f;
    if (has_bias && col_ok) {
      const T* bias = static_cast<const T*>(p.bias);
      const float2 bb = pair_to_float2<T>(*reinterpret_cast<const uint32_t*>(bias + n0 + pr));
      b0 = bb.x;
      b1 = bb.y;
      if (SWIGLU) {
        const float2 bv = pair_to_float2<T>(
            *reinterpret_cast<const uint32_t*>(bias + p.up_row0 + n0 + pr));
        bu0 = bv.x;
        bu1 = bv.y;
      }
    }
    const uint32_t part_local = smem_addr(part);
    const uint32_t ssq_local = smem_addr(ssq);
    // Tokens in batches of kBatch: every distributed-shared-memory load of a
    // batch is issued before any is consumed (remote loads are slow).
    constexpr int kBatch = 4;
    const int t_first = static_cast<int>(rank) + S * tsub;
    const int t_end = p.M < MP ? p.M : MP;
    for (int t0 = t_first; t0 < t_end; t0 += LANES * S * kBatch) {
      float2 acc[kBatch], accu[kBatch];
      float ss[kBatch];
#pragma unroll
      for (int j = 0; j < kBatch; ++j) {
        acc[j] = make_float2(0.f, 0.f);
        accu[j] = make_float2(0.f, 0.f);
        ss[j] = 0.f;
      }
      for (int s = 0; s < S; ++s) {  // fixed rank order: deterministic sums
        const uint32_t part_s = mapa_shared(part_local, s);
        const uint32_t ssq_s = mapa_shared(ssq_local, s);
        float2 v[kBatch], u[kBatch];
        float q[kBatch];
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
          const int t = t0 + j * LANES * S;
          const int tc = t < t_end ? t : t_first;  // clamp: loads stay in bounds
          v[j] = ld_shared_cluster_f32x2(part_s + (tc * C::BM + pr) * 4);
          if (SWIGLU) u[j] = ld_shared_cluster_f32x2(part_s + (tc * C::BM + 64 + pr) * 4);
          q[j] = ld_shared_cluster_f32(ssq_s + tc * 4);
        }
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
          acc[j].x += v[j].x;
          acc[j].y += v[j].y;
          if (SWIGLU) {
            accu[j].x += u[j].x;
            accu[j].y += u[j].y;
          }
          ss[j] += q[j];
        }
      }
#pragma unroll
      for (int j = 0; j < kBatch; ++j) {
        const int t = t0 + j * LANES * S;
        if (t < t_end && col_ok) {
          const float r = rsqrtf(ss[j] / static_cast<float>(p.K) + p.eps);
          T* o = obase + static_cast<int64_t>(t) * ostride;
          float y0 = acc[j].x * r + b0, y1 = acc[j].y * r + b1;
          if (SWIGLU) {
            y0 = __fdividef(y0, 1.0f + __expf(-y0)) * (accu[j].x * r + bu0);
            y1 = __fdividef(y1, 1.0f + __expf(-y1)) * (accu[j].y * r + bu1);
          }
          *reinterpret_cast<uint32_t*>(o) = float2_to_pair<T>(y0, y1);
        }
      }
    }
  }

  // Nobody leaves while a peer may still read its shared memory.  The peers'
  // remote reads have all returned (their values are already stored), so
  // the rendezvous needs no release.
  __syncwarp();
  cluster_sync_relaxed();
  if (*abort_flag) __nanosleep(20000);
  if (warp == C::WARP_MMA) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// ------------------------------------------------------------------ host side

// Clusters of `split` CTAs of this kernel that can be resident at once.
template <typename T, int MP, int STAGES, bool SWIGLU>
static int max_clusters(int split) {
  using C = DecodeCfg<MP, STAGES>;
  cudaLaunchConfig_t qc = {};
  qc.gridDim = dim3(split * 64);
  qc.blockDim = dim3(C::THREADS);
  qc.dynamicSmemBytes = C::SMEM_BYTES;
  cudaLaunchAttribute qa[1];
  qa[0].id = cudaLaunchAttributeClusterDimension;
  qa[0].val.clusterDim.x = split;
  qa[0].val.clusterDim.y = 1;
  qa[0].val.clusterDim.z = 1;
  qc.attrs = qa;
  qc.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, fused_rmsnorm_linear_decode_kernel<T, MP, STAGES, SWIGLU>,
                                     &qc) !=
      cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

// SWIGLU: pr.w = [gate; up] (pr.N = 2 * inter rows); the output has `inter`
// columns, 64 per tile.
template <typename T, int MP, int STAGES, bool SWIGLU = false>
static int launch_decode(const LinearProblem& pr, int split, cudaStream_t stream,
                         int64_t inter = 0) {
  using C = DecodeCfg<MP, STAGES>;
  auto kern = fused_rmsnorm_linear_decode_kernel<T, MP, STAGES, SWIGLU>;
  const int64_t n_out = SWIGLU ? inter : pr.N;
  const int tile_cols = SWIGLU ? C::BM / 2 : C::BM;
  const int tiles = static_cast<int>((n_out + tile_cols - 1) / tile_cols);
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return set_cuda_error("cudaGetDevice");
  static bool attr_set[kMaxDevices] = {};
  if (dev < kMaxDevices && !attr_set[dev]) {
    cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return set_cuda_error("cudaFuncSetAttribute(decode kernel)", e);
    attr_set[dev] = true;
  }
  // Largest k-split (<= the requested one) whose clusters all fit in one
  // wave: a second wave would double the time of this weight stream.
  {
    static int fits[kMaxDevices][9] = {};
    while (split > 1) {
      int& f = fits[dev < kMaxDevices ? dev : 0][split];
      if (f == 0) f = max_clusters<T, MP, STAGES, SWIGLU>(split) + 1;  // 0 = "not queried"
      if (tiles <= f - 1) break;
      --split;
    }
  }
  const CUtensorMapDataType dt = Elem16<T>::kTmaType;
  CUtensorMap tw, tx;
  int rc = encode_tmap_2d(&tw, dt, 2, pr.w, pr.K, pr.N, pr.w_row_stride, C::BK,
                          SWIGLU ? C::BM / 2 : C::BM, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = encode_tmap_2d(&tx, dt, 2, pr.x, pr.K, pr.M, pr.x_row_stride, C::BK, MP,
                      CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  DecodeParams p;
  p.M = static_cast<int32_t>(pr.M);
  p.N = static_cast<int32_t>(n_out);
  p.K = static_cast<int32_t>(pr.K);
  p.num_k_blocks = static_cast<int32_t>((pr.K + C::BK - 1) / C::BK);
  p.split = split;
  p.eps = pr.eps;
  p.bias = pr.bias;
  if (pr.parts && pr.parts->n > 1) {
    p.nparts = pr.parts->n;
    for (int i = 0; i < kMaxParts; ++i) {
      const bool used = i < pr.parts->n;
      p.part_col0[i] = used ? static_cast<int32_t>(pr.parts->col0[i]) : 0x7fffffff;
      p.part_out[i] = used ? pr.parts->out[i] : nullptr;
      p.part_stride[i] = used ? pr.parts->stride[i] : 0;
    }
  } else {
    p.nparts = 1;
    for (int i = 0; i < kMaxParts; ++i) {
      p.part_col0[i] = i == 0 ? 0 : 0x7fffffff;
      p.part_out[i] = i == 0 ? pr.out : nullptr;
      p.part_stride[i] = i == 0 ? pr.out_row_stride : 0;
    }
  }
  p.up_row0 = static_cast<int32_t>(inter);
  p.timeout_ns = wait_timeout_ns();

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(tiles * split);
  cfg.blockDim = dim3(C::THREADS);
  cfg.dynamicSmemBytes = C::SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[2];
  attrs[0].id = cudaLaunchAttributeClusterDimension;
  attrs[0].val.clusterDim.x = split;
  attrs[0].val.clusterDim.y = 1;
  attrs[0].val.clusterDim.z = 1;
  attrs[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attrs;
  cfg.numAttrs = 2;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, tw, tx, p);
  if (e != cudaSuccess) return set_cuda_error("launch fused_rmsnorm_linear_decode", e);
  return 0;
}

// k-split per W tile: as many CTAs per tile as fit one wave (<= 8, the
// portable cluster size) without splits shorter than 4 k-blocks.
int choose_decode_split(int64_t N, int64_t K, int sms) {
  const int64_t tiles = (N + 127) / 128;
  const int64_t nkb = (K + 63) / 64;
  int s = static_cast<int>(sms / (tiles > 0 ? tiles : 1));
  if (s > 8) s = 8;
  while (s > 1 && nkb / s < 4) --s;
  return s < 1 ? 1 : s;
}

template <typename T>
static int run_decode_t(const LinearProblem& pr, int split, cudaStream_t s) {
  if (pr.M <= 16) return launch_decode<T, 16, 8>(pr, split, s);
  if (pr.M <= 32) return launch_decode<T, 32, 8>(pr, split, s);
  if (pr.M <= 64) return launch_decode<T, 64, 6>(pr, split, s);
  if (pr.M <= 128) return launch_decode<T, 128, 6>(pr, split, s);
  return set_error(FRN_ERR_UNSUPPORTED, "decode kernel takes M <= 128 (got %lld)",
                   static_cast<long long>(pr.M));
}

int run_fused_linear_decode(const LinearProblem& pr, int split, cudaStream_t s) {
  if (pr.dtype == FRN_DTYPE_BF16) return run_decode_t<__nv_bfloat16>(pr, split, s);
  if (pr.dtype == FRN_DTYPE_F16) return run_decode_t<__half>(pr, split, s);
  return set_error(FRN_ERR_UNSUPPORTED, "fused RMSNorm+Linear supports bf16 and fp16 only");
}

template <typename T>
static int run_decode_swiglu_t(const LinearProblem& pr, int64_t inter, int split,
                               cudaStream_t s) {
  if (pr.M <= 16) return launch_decode<T, 16, 8, true>(pr, split, s, inter);
  if (pr.M <= 32) return launch_decode<T, 32, 8, true>(pr, split, s, inter);
  if (pr.M <= 64) return launch_decode<T, 64, 6, true>(pr, split, s, inter);
  if (pr.M <= 128) return launch_decode<T, 128, 6, true>(pr, split, s, inter);
  return set_error(FRN_ERR_UNSUPPORTED, "decode kernel takes M <= 128 (got %lld)",
                   static_cast<long long>(pr.M));
}

int run_fused_swiglu_decode(const LinearProblem& pr, int64_t inter, int split, cudaStream_t s) {
  if (pr.dtype == FRN_DTYPE_BF16) return run_decode_swiglu_t<__nv_bfloat16>(pr, inter, split, s);
  if (pr.dtype == FRN_DTYPE_F16) return run_decode_swiglu_t<__half>(pr, inter, split, s);
  return set_error(FRN_ERR_UNSUPPORTED, "fused RMSNorm+SwiGLU supports bf16 and fp16 only");
}

}  // namespace frn
