// frn_fused_linear_pair.cu -- fused RMSNorm -> Linear on SM pairs (cta_group::2).
//
// Same math as frn_fused_linear.cu; one 256 x BN output tile per CTA pair:
// tcgen05.mma.cta_group::2 with M = 256 reads A (x rows) from both CTAs'
// shared memory (128 rows each) and B (W rows) split in two halves of BN/2
// rows, so every SM loads 16 KB of x and BN*64 B of W per 64-deep k-block
// instead of 16 KB + BN*128 B: the L2 -> SM traffic per MMA halves for W.
//
// Roles (each CTA of the pair):
//   warps 0-3   epilogue: TMEM lanes of this CTA's 128 rows -> acc * inv_rms
//               + b -> one rounding -> swizzled smem block per warp -> TMA
//               tensor store (double-buffered per warp).
//   warps 4-7   TMA producers: x tile / W half-tile, each split over even and
//               odd stages (four issuing threads, because one thread keeps
//               only a few bulk-tensor loads in flight).  Both CTAs' loads
//               complete on the EVEN CTA's `full` barrier, which the even
//               CTA's x-producers arm with the bytes of the whole pair.
//   warp 8      even CTA: single-thread MMA issuer; every CTA: TMEM owner.
//               After each k-block the MMA commit is multicast to both CTAs'
//               `mma_done[stage]`; after each tile to both `tmem_full[acc]`.
//   warps 9-12  RMS reducers: once the MMA has consumed a stage, thread t
//               sums x[row t]^2 from this CTA's copy of the stage and then
//               frees the stage (empty barrier, 4 arrivals).  Only the first
//               tile of each run of same-m-block tiles is reduced; later
//               tiles reuse the cached inv_rms and just free the stages.
// The epilogue warps of both CTAs release an accumulator by arriving on the
// even CTA's `tmem_empty[acc]` (8 arrivals).
#include <cuda.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "frn_internal.h"
#include "frn_pair_common.cuh"
#include "frn_ptx.cuh"

namespace frn {

// NACC accumulators of BN columns per pair tile: NACC = 1 double-buffers the
// accumulator in TMEM (tile i's epilogue overlaps tile i+1's mainloop); NACC
// = 2 makes the tile 256 x 2*BN so one x tile feeds two W tiles (25% fewer
// L2->SM bytes per MMA) and uses the TMEM columns for that instead.
template <int BN, int STAGES, int NACC>
struct PairCfg {
  static constexpr int BM = 128;  // rows per CTA
  static constexpr int BK = 64;
  static constexpr int BN_HALF = BN / 2;
  static constexpr int TILE_N = NACC * BN;  // output columns per pair tile
  static constexpr int NBUF = NACC == 1 ? 2 : 1;  // TMEM accumulator buffers
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN_HALF * BK * 2;  // one accumulator's W half-tile
  static constexpr uint32_t PAIR_TX = 2u * (A_BYTES + NACC * B_BYTES);
  static constexpr uint32_t TMEM_COLS = (NBUF * TILE_N <= 256) ? 256u : 512u;
  static constexpr int STG_BYTES = 32 * 128;  // one warp's 32 rows x 64 columns
  static constexpr int NCHUNK = (TILE_N + 63) / 64;  // epilogue chunks of 64 columns
  static constexpr bool HALF_TAIL = TILE_N % 64 != 0;  // last chunk is 32 columns
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = OFF_A + STAGES * A_BYTES;
  static constexpr int OFF_STG = OFF_B + STAGES * NACC * B_BYTES;
  static constexpr int OFF_RMS = OFF_STG + 4 * 2 * STG_BYTES;
  static constexpr int OFF_BAR = OFF_RMS + 2 * BM * 4;
  static constexpr int NUM_BARS = 3 * STAGES + 9;
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
  static constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;
  static constexpr int EPI_WARPS = 4;
  static constexpr int RMS_WARPS = 4;
  static constexpr int WARP_PROD0 = 4;  // warps 4..7: (x | W) x (even | odd stages)
  static constexpr int WARP_MMA = 8;
  static constexpr int WARP_RMS0 = 9;
  static constexpr int THREADS = 32 * (EPI_WARPS + 5 + RMS_WARPS);
  static_assert(STAGES % 2 == 0, "stages are split between two producers per operand");
  // UMMA N for M = 256: a multiple of 16 up to 256.  The epilogue stores
  // 64-column chunks and at most one 32-column tail per tile.
  static_assert(BN % 16 == 0 && BN >= 32 && BN <= 256, "BN");
  static_assert(TILE_N % 32 == 0, "tile width must be a multiple of 32 columns");
  static_assert(NACC == 1 || NACC == 2, "NACC");
  static_assert(NBUF * TILE_N <= 512, "TMEM has 512 columns");
  static_assert(B_BYTES % 1024 == 0, "stage buffers must stay 1024-aligned");
  static_assert(OFF_STG % 1024 == 0, "staging blocks must be 1024-aligned for the 128B swizzle");
  static_assert(SMEM_BYTES <= 232448, "exceeds 227 KB of dynamic shared memory");
};

// SWIGLU (with NACC = 2): accumulator 0 holds x.W_gate^T for output columns
// [n0, n0+BN), accumulator 1 x.W_up^T for the same columns (W rows up_row0 +
// n), and the epilogue writes silu(g * inv_rms + b_g) * (u * inv_rms + b_u).
template <typename T, int BN, int STAGES, int NACC, bool SWIGLU>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(PairCfg<BN, STAGES, NACC>::THREADS, 1)
    fused_rmsnorm_linear_pair_kernel(const __grid_constant__ CUtensorMap tmap_x,
                                     const __grid_constant__ CUtensorMap tmap_w,
                                     const __grid_constant__ PairOut outm,
                                     const PairParams p) {
  using C = PairCfg<BN, STAGES, NACC>;
  static_assert(!SWIGLU || NACC == 2, "the SwiGLU epilogue pairs the two accumulators");
  constexpr int OUT_N = SWIGLU ? BN : C::TILE_N;  // output columns per pair tile
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));

  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);  // used in the even CTA
  uint64_t* mma_done = full + STAGES;
  uint64_t* empty = mma_done + STAGES;
  uint64_t* tmem_full = empty + STAGES;
  uint64_t* tmem_empty = tmem_full + 2;  // used in the even CTA
  uint64_t* rms_full = tmem_empty + 2;
  uint64_t* rms_empty = rms_full + 2;
  uint64_t* drain = rms_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile uint32_t* abort_flag = tmem_slot + 1;
  float* rms_buf = reinterpret_cast<float*>(smem + C::OFF_RMS);

  const uint32_t warp = warp_id_in_cta();
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t rank = cluster_cta_rank();  // 0 = even CTA (MMA issuer), 1 = odd
  const uint32_t pair = blockIdx.x >> 1;
  const uint32_t num_pairs = gridDim.x >> 1;

  if (warp == C::WARP_PROD0 && lane == 0) {
    prefetch_tmap(&tmap_x);
    prefetch_tmap(&tmap_w);
    for (int i = 0; i < outm.nparts; ++i) prefetch_tmap(&outm.map[i]);
    if (OUT_N % 64 != 0) prefetch_tmap(&outm.half);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&mma_done[s], 1);
      mbar_init(&empty[s], C::RMS_WARPS);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tmem_full[a], 1);
      mbar_init(&tmem_empty[a], 2 * C::EPI_WARPS);  // only the first NBUF are used
      mbar_init(&rms_full[a], C::RMS_WARPS);
      mbar_init(&rms_empty[a], C::EPI_WARPS);
    }
    mbar_init(drain, 1);
    *abort_flag = 0u;
    fence_mbarrier_init();
  }
  if (warp == C::WARP_MMA) {
    tmem_alloc_pair(tmem_slot, C::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  // Both CTAs' barriers must be initialised before either signals the other.
  // __syncthreads publishes this CTA's inits and TMEM slot to its own
  // threads; the peer's inits were released cluster-wide by its
  // fence.mbarrier_init, so the cluster rendezvous itself is relaxed.
  __syncthreads();
  cluster_sync_relaxed();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // Each pair owns a contiguous run [t_begin, t_end) of the tiles in
  // m-block-major order, so consecutive tiles of a pair mostly share their
  // m-block and inv_rms is reduced once per run rather than once per tile.
  const int num_tiles = p.num_m_blocks * p.num_n_blocks;
  const int tiles_base = num_tiles / static_cast<int>(num_pairs);
  const int tiles_rem = num_tiles % static_cast<int>(num_pairs);
  const int t_begin = static_cast<int>(pair) * tiles_base +
                      min(static_cast<int>(pair), tiles_rem);
  const int t_end = t_begin + tiles_base + (static_cast<int>(pair) < tiles_rem ? 1 : 0);
  const int nkb = p.num_k_blocks;
  const uint64_t to = p.timeout_ns;
  // Let the next kernel in the stream get scheduled now: its CTAs take SMs as
  // ours retire and run their set-up while we finish; its griddepcontrol.wait
  // still orders all of its global accesses after this whole grid.
  griddep_launch_dependents();

  if (warp >= C::WARP_PROD0 && warp < C::WARP_PROD0 + 4) {
    // Four issuing threads: a single thread keeps only a few bulk-tensor loads
    // in flight, so x and W loads are split by operand and by stage parity.
    if (lane == 0) {
      const uint32_t pid = warp - C::WARP_PROD0;
      const bool is_a = (pid & 1u) == 0;
      const uint32_t parity_sel = pid >> 1;  // this thread fills stages with s % 2 == parity_sel
      if (t_begin < t_end) {
        // While the preceding grid drains, pull this thread's first ring of
        // tiles into L2 so the first loads after the wait do not go to HBM.
        const int pm0 = (t_begin / p.num_n_blocks) * 2 * C::BM + rank * C::BM;
        const int pn0 = (t_begin % p.num_n_blocks) * OUT_N + rank * C::BN_HALF;
        for (int kb = static_cast<int>(parity_sel); kb < nkb && kb < STAGES; kb += 2) {
          if (is_a) {
            tma_prefetch_2d(&tmap_x, kb * C::BK, pm0);
          } else {
#pragma unroll
            for (int j = 0; j < NACC; ++j)
              tma_prefetch_2d(&tmap_w, kb * C::BK,
                              SWIGLU ? (j == 0 ? pn0 : p.up_row0 + pn0) : pn0 + j * BN);
          }
        }
      }
      griddep_wait();
      const bool arms = is_a && rank == 0;
      uint32_t stage = 0, phase = 0;
      for (int t = t_begin; t < t_end; ++t) {
        const int m0 = (t / p.num_n_blocks) * 2 * C::BM + rank * C::BM;
        const int n0 = (t % p.num_n_blocks) * OUT_N + rank * C::BN_HALF;
        bool ok = true;
        for (int kb = 0; kb < nkb; ++kb) {
          if ((stage & 1u) == parity_sel) {
            if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, to)) { ok = false; break; }
            const uint32_t leader_full = mapa_shared(smem_addr(&full[stage]), 0);
            if (arms) mbar_arrive_expect_tx(&full[stage], C::PAIR_TX);
            if (is_a)
              tma_load_2d_pair(smem + C::OFF_A + stage * C::A_BYTES, &tmap_x, leader_full,
                               kb * C::BK, m0);
            else
#pragma unroll
              for (int j = 0; j < NACC; ++j)
                tma_load_2d_pair(smem + C::OFF_B + (stage * NACC + j) * C::B_BYTES, &tmap_w,
                                 leader_full, kb * C::BK,
                                 SWIGLU ? (j == 0 ? n0 : p.up_row0 + n0) : n0 + j * BN);
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
      }
    }
  } else if (warp == C::WARP_MMA) {
    if (rank == 0 && lane == 0) {
      const uint32_t idesc = make_idesc_f16(Elem16<T>::kUmmaFormat, 2 * C::BM, BN);
      uint32_t stage = 0, phase = 0;
      int i = 0;
      bool ok = true;
      for (int t = t_begin; t < t_end && ok; ++t, ++i) {
        const uint32_t acc = i % C::NBUF, acc_phase = (i / C::NBUF) & 1;
        if (!mbar_wait_cluster(&tmem_empty[acc], acc_phase ^ 1u, abort_flag, to)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * C::TILE_N;
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, to)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_addr(smem + C::OFF_A + stage * C::A_BYTES);
          const uint32_t b_addr = smem_addr(smem + C::OFF_B + stage * NACC * C::B_BYTES);
#pragma unroll
          for (int k = 0; k < C::BK / 16; ++k) {
#pragma unroll
            for (int j = 0; j < NACC; ++j)
              umma_f16_ss_pair(d_tmem + j * BN, make_smem_desc_k_sw128(a_addr + k * 32),
                               make_smem_desc_k_sw128(b_addr + j * C::B_BYTES + k * 32), idesc,
                               (kb > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit_pair_mc(&mma_done[stage], 0x3);
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        umma_commit_pair_mc(&tmem_full[acc], 0x3);
      }
      umma_commit_pair_mc(drain, 0x1);
      uint32_t zero = 0;
      mbar_wait(drain, 0, &zero, to);
    }
  } else if (warp >= C::WARP_RMS0) {
    // inv_rms depends only on the m-block, so it is reduced on the first tile
    // of each run of consecutive tiles with the same m-block (a "generation")
    // and kept in rms_buf[gen & 1] until the epilogue has finished the run.
    const int r = static_cast<int>(threadIdx.x) - C::WARP_RMS0 * 32;  // row in this CTA's half
    const float inv_k = 1.0f / static_cast<float>(p.K);
    uint32_t stage = 0, phase = 0;
    int gen = -1, cur_m = -1;
    bool ok = true;
    for (int t = t_begin; t < t_end && ok; ++t) {
      const int mb = t / p.num_n_blocks;
      const bool first = (mb != cur_m);
      if (first) { ++gen; cur_m = mb; }
      float ss0 = 0.f, ss1 = 0.f;
      for (int kb = 0; kb < nkb; ++kb) {
        if (!mbar_wait(&mma_done[stage], phase, abort_flag, to)) { ok = false; break; }
        const uint32_t row = smem_addr(smem + C::OFF_A + stage * C::A_BYTES) + r * 128;
        if (first)
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const uint4 v = ld_shared_v4(row + ((q ^ (r & 7)) << 4));
          const float2 f0 = pair_to_float2<T>(v.x), f1 = pair_to_float2<T>(v.y);
          const float2 f2 = pair_to_float2<T>(v.z), f3 = pair_to_float2<T>(v.w);
          ss0 = fmaf(f0.x, f0.x, ss0); ss1 = fmaf(f0.y, f0.y, ss1);
          ss0 = fmaf(f1.x, f1.x, ss0); ss1 = fmaf(f1.y, f1.y, ss1);
          ss0 = fmaf(f2.x, f2.x, ss0); ss1 = fmaf(f2.y, f2.y, ss1);
          ss0 = fmaf(f3.x, f3.x, ss0); ss1 = fmaf(f3.y, f3.y, ss1);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[stage]);
        if (++stage == STAGES) { stage = 0; phase ^= 1u; }
      }
      if (!ok || !first) continue;
      const uint32_t g = static_cast<uint32_t>(gen);
      if (!mbar_wait(&rms_empty[g & 1], ((g >> 1) & 1) ^ 1u, abort_flag, to)) break;
      rms_buf[(g & 1) * C::BM + r] = rsqrtf((ss0 + ss1) * inv_k + p.eps);
      __syncwarp();
      if (lane == 0) mbar_arrive(&rms_full[g & 1]);
    }
  } else {
    // Epilogue: warp q owns TMEM lanes [32q, 32q+32) = rows of this CTA's half.
    const uint32_t q = warp;
    const bool has_bias = p.bias != nullptr;
    const T* bias = static_cast<const T*>(p.bias);
    const uint32_t leader_tmem_empty0 = mapa_shared(smem_addr(&tmem_empty[0]), 0);
    griddep_wait();
    uint32_t nst = 0;  // chunks this warp has staged: staging buffer nst & 1
    int i = 0;
    int gen = -1, cur_m = -1;
    float inv_rms = 0.f;
    for (int t = t_begin; t < t_end; ++t, ++i) {
      const uint32_t acc = i % C::NBUF, acc_phase = (i / C::NBUF) & 1;
      const int mb = t / p.num_n_blocks;
      const int row = mb * 2 * C::BM + rank * C::BM + q * 32 + lane;
      const int n0 = (t % p.num_n_blocks) * OUT_N;
      const bool first = (mb != cur_m);
      const bool last = (t + 1 >= t_end) || ((t + 1) / p.num_n_blocks != mb);
      if (first) { ++gen; cur_m = mb; }
      const uint32_t g = static_cast<uint32_t>(gen);
      if (!mbar_wait(&tmem_full[acc], acc_phase, abort_flag, to)) break;
      if (first) {
        if (!mbar_wait(&rms_full[g & 1], (g >> 1) & 1, abort_flag, to)) break;
        inv_rms = rms_buf[(g & 1) * C::BM + q * 32 + lane];
      }
      tc_fence_after();
      if (last) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&rms_empty[g & 1]);
      }
      const int row_base = row - static_cast<int>(lane);  // first row of this warp
      const bool reuse_acc = t + C::NBUF < t_end;
      if constexpr (SWIGLU) {
        constexpr int NCH = (BN + 63) / 64;
        constexpr bool HALF = BN % 64 != 0;
        const uint32_t tg = tmem_base + ((q * 32u) << 16);  // gate accumulator
        const uint32_t tu = tg + BN;                        // up accumulator
#pragma unroll 1
        for (int c = 0; c < NCH; ++c, ++nst) {
          const bool half = HALF && c == NCH - 1;
          const int col0 = n0 + c * 64;
          uint8_t* sbp = smem + C::OFF_STG + (q * 2 + (nst & 1u)) * C::STG_BYTES;
          const uint32_t sb = smem_addr(sbp);
          if (lane == 0) bulk_wait_group_read<1>();
          __syncwarp();
#pragma unroll 1
          for (int h = 0; h < (half ? 1 : 2); ++h) {
            // 32 output columns: gate and up accumulators side by side.
            const int colh = col0 + h * 32;
            uint4 bg[4], bu[4];
            if (has_bias) {
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const bool in = colh + j * 8 < p.N;
                bg[j] = in ? ld_global_nc_v4(bias + colh + j * 8) : make_uint4(0u, 0u, 0u, 0u);
                bu[j] = in ? ld_global_nc_v4(bias + p.up_row0 + colh + j * 8)
                           : make_uint4(0u, 0u, 0u, 0u);
              }
            }
            uint32_t gv[32], uv[32];
            tmem_ld_32x32b_x32(tg + c * 64 + h * 32, gv);
            tmem_ld_32x32b_x32(tu + c * 64 + h * 32, uv);
            tmem_ld_wait();
            if (c == NCH - 1 && (half || h == 1) && reuse_acc) {
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive_cluster_relaxed(leader_tmem_empty0);
            }
            if (half) {
              if (has_bias) stage_swiglu_rows<T, 4, true>(gv, uv, inv_rms, bg, bu, sb, lane, 0);
              else stage_swiglu_rows<T, 4, false>(gv, uv, inv_rms, bg, bu, sb, lane, 0);
            } else {
              if (has_bias) stage_swiglu_rows<T, 8, true>(gv, uv, inv_rms, bg, bu, sb, lane, h * 4);
              else stage_swiglu_rows<T, 8, false>(gv, uv, inv_rms, bg, bu, sb, lane, h * 4);
            }
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(half ? &outm.half : &outm.map[0], sbp, col0, row_base);
            bulk_commit_group();
          }
        }
        continue;
      }
      pair_store_linear_tile<T, C::TILE_N>(smem + C::OFF_STG + q * 2 * C::STG_BYTES, lane,
                                            tmem_base + acc * C::TILE_N + ((q * 32u) << 16),
                                            n0, row_base, inv_rms, has_bias ? bias : nullptr, p.N,
                                            outm, nst, reuse_acc, leader_tmem_empty0 + acc * 8);
    }
    // The staging blocks must not be released while a store still reads them;
    // the global writes themselves are complete when the grid is.
    if (lane == 0) bulk_wait_group_read<0>();
  }

  // Every thread of both CTAs gets here (all waits are bounded), so the pair
  // never leaves with the other CTA still reading its smem or barriers.  Each
  // cross-CTA signal (pair loads, multicast commits, accumulator releases) has
  // been waited for by its target by now, so the rendezvous is relaxed.
  __syncwarp();
  tc_fence_before();
  cluster_sync_relaxed();
  if (*abort_flag) {
    // A wait expired: give in-flight bulk copies into this CTA time to land.
    __nanosleep(20000);
  }
  if (warp == C::WARP_MMA) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
  }
}

// ------------------------------------------------------------------ host side

// SWIGLU: pr.w holds [gate; up] (pr.N = 2 * inter rows) and the output has
// `inter` columns.
template <typename T, int BN, int STAGES, int NACC, bool SWIGLU = false>
static int launch_pair(const LinearProblem& pr, cudaStream_t stream, int64_t inter = 0) {
  using C = PairCfg<BN, STAGES, NACC>;
  constexpr int OUT_N = SWIGLU ? BN : C::TILE_N;
  const int64_t n_out = SWIGLU ? inter : pr.N;
  auto kern = fused_rmsnorm_linear_pair_kernel<T, BN, STAGES, NACC, SWIGLU>;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return set_cuda_error("cudaGetDevice");
  static int max_pairs[kMaxDevices] = {};
  if (dev < kMaxDevices && max_pairs[dev] == 0) {
    cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
    if (e != cudaSuccess) return set_cuda_error("cudaFuncSetAttribute(pair kernel)", e);
    cudaLaunchConfig_t qc = {};
    qc.gridDim = dim3(2 * 74);
    qc.blockDim = dim3(C::THREADS);
    qc.dynamicSmemBytes = C::SMEM_BYTES;
    cudaLaunchAttribute qa[1];
    qa[0].id = cudaLaunchAttributeClusterDimension;
    qa[0].val.clusterDim.x = 2;
    qa[0].val.clusterDim.y = 1;
    qa[0].val.clusterDim.z = 1;
    qc.attrs = qa;
    qc.numAttrs = 1;
    int clusters = 0;
    e = cudaOccupancyMaxActiveClusters(&clusters, kern, &qc);
    if (e != cudaSuccess || clusters <= 0) {
      cudaGetLastError();
      clusters = sm_count(dev) / 2;
    }
    max_pairs[dev] = clusters;
  }
  const int pairs_avail = dev < kMaxDevices ? max_pairs[dev] : sm_count(dev) / 2;

  const CUtensorMapDataType dt = Elem16<T>::kTmaType;
  CUtensorMap tx, tw;
  int rc = encode_tmap_2d(&tx, dt, 2, pr.x, pr.K, pr.M, pr.x_row_stride, C::BK, C::BM,
                          CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = encode_tmap_2d(&tw, dt, 2, pr.w, pr.K, pr.N, pr.w_row_stride, C::BK, C::BN_HALF,
                      CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  // Output: one warp's [32 rows x 64 columns] block per store (128B swizzle),
  // and [32 x 32] with the 64B swizzle for a tile whose last chunk is 32 wide.
  PairOut outm;
  if (SWIGLU && pr.parts && pr.parts->n > 1)
    return set_error(FRN_ERR_UNSUPPORTED, "split output is for the linear op only");
  rc = build_pair_out(pr, n_out, OUT_N % 64 != 0, &outm);
  if (rc) return rc;

  PairParams p;
  p.M = static_cast<int32_t>(pr.M);
  p.N = static_cast<int32_t>(n_out);
  p.K = static_cast<int32_t>(pr.K);
  p.num_m_blocks = static_cast<int32_t>((pr.M + 2 * C::BM - 1) / (2 * C::BM));
  p.num_n_blocks = static_cast<int32_t>((n_out + OUT_N - 1) / OUT_N);
  p.num_k_blocks = static_cast<int32_t>((pr.K + C::BK - 1) / C::BK);
  p.eps = pr.eps;
  p.bias = pr.bias;
  p.out = pr.out;
  p.out_row_stride = pr.out_row_stride;
  p.up_row0 = static_cast<int32_t>(inter);
  p.timeout_ns = wait_timeout_ns();
  const int tiles = p.num_m_blocks * p.num_n_blocks;
  const int pairs = tiles < pairs_avail ? tiles : pairs_avail;

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs);
  cfg.blockDim = dim3(C::THREADS);
  cfg.dynamicSmemBytes = C::SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[1];
  attrs[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attrs;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, tx, tw, outm, p);
  if (e != cudaSuccess) return set_cuda_error("launch fused_rmsnorm_linear_pair", e);
  return 0;
}

// Pair-tile choice.  Per pair tile of 256 x (NACC*BN) over nkb 64-deep
// k-blocks, in SM cycles:
//   mma  = nkb * 2 * NACC * BN                 (two SMs, 4096 MAC/clk each)
//   feed = nkb * (16 KB + NACC * BN * 64 B) / 60 B/clk   (measured L2->SM
//          ceiling per SM when every SM loads tiles)
//   epi  = 128 * NACC * BN * 2 B / 26 B/clk    (epilogue drain per CTA)
// A tile costs max(mma, feed); with NACC = 1 the epilogue overlaps the next
// tile and only the last one is exposed, with NACC = 2 every epilogue is.
// The busiest pair runs ceil(tiles / pairs) tiles.
PairChoice choose_pair_tiling(int64_t M, int64_t N, int64_t K, int pairs, bool tile64) {
  const double mb = static_cast<double>((M + 255) / 256);
  const double nkb = static_cast<double>((K + 63) / 64);
  static const PairChoice cands[] = {{256, 1}, {224, 1}, {192, 1}, {160, 1}, {128, 1},
                                     {256, 2}, {224, 2}, {192, 2}, {176, 2}, {128, 2}};
  double best = 1e300;
  PairChoice pick = {256, 1};
  for (const PairChoice& c : cands) {
    if (tile64 && (c.nacc * c.bn) % 64 != 0) continue;
    const double tn = static_cast<double>(c.nacc * c.bn);
    const double tiles = mb * std::ceil(static_cast<double>(N) / tn);
    const double per_pair = std::ceil(tiles / pairs);
    const double mma = nkb * 2.0 * tn;
    const double feed = nkb * (16384.0 + tn * 64.0) / 60.0;
    const double epi = 128.0 * tn * 2.0 / 26.0;
    const double tile = (mma > feed ? mma : feed) + (c.nacc == 2 ? epi : 0.0);
    const double total = per_pair * tile + (c.nacc == 1 ? epi : 0.0);
    if (total < best * 0.999) { best = total; pick = c; }
  }
  return pick;
}

template <typename T>
static int run_pair_t(const LinearProblem& pr, PairChoice c, cudaStream_t s) {
  if (c.nacc == 2) {
    switch (c.bn) {
      case 256: return launch_pair<T, 256, 4, 2>(pr, s);
      case 224: return launch_pair<T, 224, 4, 2>(pr, s);
      case 192: return launch_pair<T, 192, 4, 2>(pr, s);
      case 176: return launch_pair<T, 176, 4, 2>(pr, s);
      case 128: return launch_pair<T, 128, 6, 2>(pr, s);
      default: break;
    }
  } else {
    switch (c.bn) {
      case 256: return launch_pair<T, 256, 6, 1>(pr, s);
      case 224: return launch_pair<T, 224, 6, 1>(pr, s);
      case 192: return launch_pair<T, 192, 6, 1>(pr, s);
      case 160: return launch_pair<T, 160, 6, 1>(pr, s);
      case 128: return launch_pair<T, 128, 8, 1>(pr, s);
      default: break;
    }
  }
  return set_error(FRN_ERR_INVALID_ARGUMENT, "unsupported pair tiling %d x %d", c.nacc, c.bn);
}

int run_fused_linear_pair(const LinearProblem& pr, PairChoice c, cudaStream_t s) {
  if (pr.dtype == FRN_DTYPE_BF16) return run_pair_t<__nv_bfloat16>(pr, c, s);
  if (pr.dtype == FRN_DTYPE_F16) return run_pair_t<__half>(pr, c, s);
  return set_error(FRN_ERR_UNSUPPORTED, "fused RMSNorm+Linear supports bf16 and fp16 only");
}

// SwiGLU output-tile width (tile = 256 rows x bn output columns over two
// bn-wide accumulators, gate and up): the cost model of choose_pair_tiling
// with 2*bn columns of MMA per tile and every epilogue exposed.
int choose_swiglu_bn(int64_t M, int64_t inter, int64_t K, int pairs) {
  const double mb = static_cast<double>((M + 255) / 256);
  const double nkb = static_cast<double>((K + 63) / 64);
  static const int cands[] = {256, 224, 192, 128};
  double best = 1e300;
  int pick = 256;
  for (int bn : cands) {
    const double tiles = mb * std::ceil(static_cast<double>(inter) / bn);
    const double per_pair = std::ceil(tiles / pairs);
    const double mma = nkb * 2.0 * (2.0 * bn);
    const double feed = nkb * (16384.0 + 2.0 * bn * 64.0) / 60.0;
    const double epi = 128.0 * bn * 2.0 / 26.0;
    const double total = per_pair * ((mma > feed ? mma : feed) + epi);
    if (total < best * 0.999) { best = total; pick = bn; }
  }
  return pick;
}

template <typename T>
static int run_swiglu_t(const LinearProblem& pr, int64_t inter, int bn, cudaStream_t s) {
  switch (bn) {
    case 256: return launch_pair<T, 256, 4, 2, true>(pr, s, inter);
    case 224: return launch_pair<T, 224, 4, 2, true>(pr, s, inter);
    case 192: return launch_pair<T, 192, 4, 2, true>(pr, s, inter);
    case 128: return launch_pair<T, 128, 6, 2, true>(pr, s, inter);
    default: break;
  }
  return set_error(FRN_ERR_INVALID_ARGUMENT, "unsupported SwiGLU tile width %d", bn);
}

int run_fused_swiglu_pair(const LinearProblem& pr, int64_t inter, int bn, cudaStream_t s) {
  if (pr.dtype == FRN_DTYPE_BF16) return run_swiglu_t<__nv_bfloat16>(pr, inter, bn, s);
  if (pr.dtype == FRN_DTYPE_F16) return run_swiglu_t<__half>(pr, inter, bn, s);
  return set_error(FRN_ERR_UNSUPPORTED, "fused RMSNorm+SwiGLU supports bf16 and fp16 only");
}

}  // namespace frn
