// frn_fused_linear_ts.cu -- SM-pair fused RMSNorm -> Linear with x held in
// tensor memory, for K <= 512 (Kimi kv_b: K = 512).
//
// The shared-memory port (128 B/clk per SM) carries, for every k-block of the
// smem-operand pair kernel, the TMA writes of x and W plus the MMA's operand
// reads of both; at 224-256 column tiles that is more than the port gives and
// the tensor pipe waits.  Here each CTA's 128 x K slice of x goes into TMEM
// once per run of same-m-block tiles (TMA -> smem -> tcgen05.cp, while four
// warps sum x^2 from the same smem) and the MMA reads A from TMEM
// (tcgen05.mma ... [a_tmem]), so per k-block shared memory carries W only.
// K <= 512 keeps x in TMEM columns [0, 256); two 128-column accumulators fill
// columns [256, 512).
//
// Work split: the output columns of each 256-row m-block are cut into units
// of 32 columns (64 for split outputs), and each pair owns a contiguous
// range of units (host-computed table), walked as tiles of up to 128
// columns; the last tile of a range may be narrower (any multiple of 32 is a
// valid MMA width), so the busiest pair carries ceil(units / pairs) units
// rather than a whole extra tile.
//
// Two MMA pipelines.  One thread can issue a tcgen05.mma only about every
// 115 clocks whatever the width, while a 256 x 128 pair MMA is 64 clocks of
// tensor work, so a single issuer keeps the pipe ~55% busy on 128-column
// tiles.  Tiles therefore alternate between two issuers, each with its own W
// ring and its own 128-column accumulator, and run concurrently against the
// same x in TMEM; together they keep the tensor pipe full.
//
// Roles (each CTA of the pair, 384 threads = 3 warps per SM sub-partition,
// so 168 registers a thread for the register-resident epilogue):
//   warps 0-3   epilogue: tiles in order; TMEM accumulator -> registers
//               (acc * inv_rms + b, rounded) -> release the accumulator to
//               its pipeline -> swizzled smem -> TMA tensor store
//   warps 4, 5  W loaders of pipeline 0 / 1 (tiles 0, 2, 4, ... / 1, 3, ...);
//               both CTAs' halves complete on the even CTA's `w_full`.
//               Warp 4 also loads x at the start of each run (groups of four
//               k-blocks, completing on the even CTA's `x_full`)
//   warp 6      even CTA: MMA issuer of pipeline 0, and x copier: at each
//               run start, after `x_free` (both issuers are done with the
//               previous run's x), tcgen05.cp of every x k-block into TMEM,
//               each followed by a commit multicast to `x_ready[kb]`;
//               every CTA: TMEM owner
//   warp 7      even CTA: MMA issuer of pipeline 1
//   warps 8-11  RMS: per run, after `x_ready[kb]` thread t sums x[row t]^2
//               from this CTA's smem copy of the k-block, frees each x group
//               (`x_empty`), and publishes inv_rms for the epilogue
// Every cross-CTA arrival is waited for by its target before the pair exits
// (the W loaders drain the last `w_empty` phases, the RMS warps see every
// `x_ready`, `x_free` is committed only when another run follows), so the
// exit rendezvous needs no release.
//
// Measured: correct for every shape tested, but slower than the smem-operand
// pair kernel at the Kimi shapes (kv_b 16.2 vs 12.7 us, 4096-token kv_b 71
// vs 56 us), so it is an explicit choice (FRN_KERNEL_PAIR_TS), not AUTO.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "frn_internal.h"
#include "frn_pair_common.cuh"
#include "frn_ptx.cuh"

namespace frn {

constexpr int kTsMaxPairs = 128;

// Pair p owns units [u0[p], u0[p+1]) of the m-block-major unit order.
struct TsSchedule {
  int32_t u0[kTsMaxPairs + 1];
};

struct TsParams {
  int32_t M, N, K;
  int32_t num_k_blocks;  // of 64
  int32_t units_per_mb;  // ceil(N / unit_cols)
  int32_t unit_cols;     // 32, or 64 for split outputs
  int32_t tile_units;    // 128 / unit_cols
  float eps;
  const void* bias;
  uint64_t timeout_ns;
};

template <int WP>
struct TsCfg {
  static constexpr int BM = 128;  // rows per CTA
  static constexpr int BK = 64;
  static constexpr int BN = 128;  // widest tile
  static constexpr int BN_HALF = BN / 2;
  static constexpr int MAX_KB = 8;  // K <= 512: x fills TMEM columns [0, 256)
  static constexpr int XG_KB = 4;   // x k-blocks per load group (one 3-D load of 64 KB)
  static constexpr int MAX_XG = MAX_KB / XG_KB;
  static constexpr int WS_KB = 2;   // W k-blocks per ring slot (one 3-D load of 16 KB)
  static constexpr uint32_t ACC_COL0 = 256;  // pipeline p accumulates at 256 + 128 p
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr int A_BYTES = BM * BK * 2;       // one x k-block of this CTA
  static constexpr int B_BYTES = BN_HALF * BK * 2;  // one W k-block of a half-tile
  static constexpr int WSLOT_BYTES = WS_KB * B_BYTES;
  static constexpr int STG_BYTES = 32 * 128;
  static constexpr int OFF_X = 0;
  static constexpr int OFF_W = OFF_X + MAX_KB * A_BYTES;
  static constexpr int OFF_STG = OFF_W + 2 * WP * WSLOT_BYTES;
  static constexpr int OFF_RMS = OFF_STG + 4 * 2 * STG_BYTES;
  static constexpr int OFF_BAR = OFF_RMS + 2 * BM * 4;
  static constexpr int NUM_BARS = 2 * MAX_XG + 4 * WP + MAX_KB + 1 + 8 + 2;
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
  static constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;
  static constexpr int WARP_WLOAD0 = 4, WARP_MMA0 = 6, WARP_MMA1 = 7, WARP_RMS0 = 8;
  static constexpr int THREADS = 32 * 12;
  static_assert(OFF_W % 1024 == 0 && OFF_STG % 1024 == 0, "1024-aligned swizzled buffers");
  static_assert(SMEM_BYTES <= 232448, "exceeds 227 KB of dynamic shared memory");
};

// Tile at unit u of a pair whose range ends at u_end: m-block, first output
// column, width in columns; returns the unit after the tile.
struct TsTile {
  int mb, n0, width;
};
__device__ __forceinline__ int ts_tile(const TsParams& p, int u, int u_end, TsTile& t) {
  const int mb = u / p.units_per_mb;
  const int cu = u - mb * p.units_per_mb;
  int w = p.tile_units;
  w = min(w, u_end - u);
  w = min(w, p.units_per_mb - cu);
  t.mb = mb;
  t.n0 = cu * p.unit_cols;
  t.width = w * p.unit_cols;
  return u + w;
}

// TMEM -> registers for one 64-column chunk (32 columns if `half`): the
// lane's row, scaled by inv_rms, biased and rounded once, as 32 (16) packed
// pairs of T.
template <typename T>
__device__ __forceinline__ void ts_drain_chunk(uint32_t taddr, bool half, int col0,
                                               float inv_rms, const T* bias, int N,
                                               uint32_t (&pk)[32]) {
  uint32_t v[64];
  tmem_ld_32x32b_x32(taddr, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
  if (!half) tmem_ld_32x32b_x32(taddr + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
  tmem_ld_wait();
#pragma unroll
  for (int g = 0; g < 8; ++g) {
    if (g < 4 || !half) {
      uint4 b = make_uint4(0u, 0u, 0u, 0u);
      if (bias != nullptr && col0 + g * 8 < N) b = ld_global_nc_v4(bias + col0 + g * 8);
      const float2 b0 = pair_to_float2<T>(b.x), b1 = pair_to_float2<T>(b.y);
      const float2 b2 = pair_to_float2<T>(b.z), b3 = pair_to_float2<T>(b.w);
      pk[g * 4 + 0] = float2_to_pair<T>(fmaf(__uint_as_float(v[g * 8 + 0]), inv_rms, b0.x),
                                        fmaf(__uint_as_float(v[g * 8 + 1]), inv_rms, b0.y));
      pk[g * 4 + 1] = float2_to_pair<T>(fmaf(__uint_as_float(v[g * 8 + 2]), inv_rms, b1.x),
                                        fmaf(__uint_as_float(v[g * 8 + 3]), inv_rms, b1.y));
      pk[g * 4 + 2] = float2_to_pair<T>(fmaf(__uint_as_float(v[g * 8 + 4]), inv_rms, b2.x),
                                        fmaf(__uint_as_float(v[g * 8 + 5]), inv_rms, b2.y));
      pk[g * 4 + 3] = float2_to_pair<T>(fmaf(__uint_as_float(v[g * 8 + 6]), inv_rms, b3.x),
                                        fmaf(__uint_as_float(v[g * 8 + 7]), inv_rms, b3.y));
    }
  }
}

// Registers -> this warp's swizzled smem block (double-buffered at stg +
// (nst % 2) * 4 KB, the layouts of stage_rows_swizzled) -> TMA tensor store
// through the output part's map, which clips rows >= M and columns >= N.
template <typename T>
__device__ __forceinline__ void ts_store_chunk(uint8_t* stg, uint32_t lane,
                                               const uint32_t (&pk)[32], bool half, int col0,
                                               int row_base, const PairOut& outm,
                                               uint32_t& nst) {
  uint8_t* sbp = stg + (nst & 1u) * 4096;
  const uint32_t sb = smem_addr(sbp);
  // The TMA store issued two chunks ago read this buffer.
  if (lane == 0) bulk_wait_group_read<1>();
  __syncwarp();
  if (half) {
#pragma unroll
    for (int j = 0; j < 4; ++j)
      st_shared_v4(sb + lane * 64u + ((static_cast<uint32_t>(j) ^ ((lane >> 1) & 3u)) << 4),
                   pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j)
      st_shared_v4(sb + lane * 128u + ((static_cast<uint32_t>(j) ^ (lane & 7u)) << 4),
                   pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    // Split outputs cut tiles at 64-column units, so a chunk never straddles
    // two parts.
    int pi = 0;
    while (pi + 1 < outm.nparts && col0 >= outm.col0[pi + 1]) ++pi;
    tma_store_2d(half ? &outm.half : &outm.map[pi], sbp, col0 - outm.col0[pi], row_base);
    bulk_commit_group();
  }
  ++nst;
}

// Epilogue of one tile for a warp whose TMEM lane quarter holds rows
// row_base .. row_base+31 of this CTA (taddr points at that quarter of the
// tile's accumulator).  The tile's `width` columns (<= 128, a multiple of 32)
// are drained into registers and the accumulator is released before anything
// is stored, so the pipeline's next MMAs overlap the staging and the stores.
template <typename T>
__device__ __forceinline__ void ts_epilogue_tile(uint8_t* stg, uint32_t lane, uint32_t taddr,
                                                 int n0, int row_base, float inv_rms,
                                                 const T* bias, int N, const PairOut& outm,
                                                 uint32_t& nst, bool release_acc,
                                                 uint32_t tmem_empty_remote, int width) {
  const bool two = width > 64;
  const bool half1 = two && (width & 63) != 0;  // second chunk is 32 wide
  const bool half0 = !two && width == 32;       // the only chunk is 32 wide
  uint32_t pk0[32], pk1[32];
  ts_drain_chunk<T>(taddr, half0, n0, inv_rms, bias, N, pk0);
  if (two) ts_drain_chunk<T>(taddr + 64, half1, n0 + 64, inv_rms, bias, N, pk1);
  if (release_acc) {
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive_cluster_relaxed(tmem_empty_remote);
  }
  ts_store_chunk<T>(stg, lane, pk0, half0, n0, row_base, outm, nst);
  if (two) ts_store_chunk<T>(stg, lane, pk1, half1, n0 + 64, row_base, outm, nst);
}

template <typename T, int WP>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(TsCfg<WP>::THREADS, 1)
    fused_rmsnorm_linear_ts_kernel(const __grid_constant__ CUtensorMap tmap_x,
                                   const __grid_constant__ CUtensorMap tmap_x3,
                                   const __grid_constant__ CUtensorMap tmap_w,
                                   const __grid_constant__ CUtensorMap tmap_w3,
                                   const __grid_constant__ PairOut outm,
                                   const __grid_constant__ TsSchedule sched,
                                   const TsParams p) {
  using C = TsCfg<WP>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));

  uint64_t* x_full = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);  // [x group], even CTA
  uint64_t* x_empty = x_full + C::MAX_XG;                            // [x group]
  uint64_t* w_full = x_empty + C::MAX_XG;  // [pipeline][slot], used in the even CTA
  uint64_t* w_empty = w_full + 2 * WP;     // [pipeline][slot]
  uint64_t* x_ready = w_empty + 2 * WP;    // [k-block]
  uint64_t* x_free = x_ready + C::MAX_KB;  // used in the even CTA
  uint64_t* tmem_full = x_free + 1;      // [pipeline]
  uint64_t* tmem_empty = tmem_full + 2;  // [pipeline], used in the even CTA
  uint64_t* rms_full = tmem_empty + 2;
  uint64_t* rms_empty = rms_full + 2;
  uint64_t* drain = rms_empty + 2;  // [pipeline], used in the even CTA
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile uint32_t* abort_flag = tmem_slot + 1;
  float* rms_buf = reinterpret_cast<float*>(smem + C::OFF_RMS);

  const uint32_t warp = warp_id_in_cta();
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t rank = cluster_cta_rank();  // 0 = even CTA (MMA issuers), 1 = odd
  const uint32_t pair = blockIdx.x >> 1;
  const int u_begin = sched.u0[pair];
  const int u_end = sched.u0[pair + 1];
  const int nkb = p.num_k_blocks;
  const int full_kb = p.K / C::BK;  // whole k-blocks: the 3-D views address only these
  const int n_xg = (nkb + C::XG_KB - 1) / C::XG_KB;
  const int n_ws = (nkb + C::WS_KB - 1) / C::WS_KB;  // W slots per tile
  const uint64_t to = p.timeout_ns;

  if (warp == C::WARP_WLOAD0 && lane == 0) {
    prefetch_tmap(&tmap_x);
    prefetch_tmap(&tmap_x3);
    prefetch_tmap(&tmap_w);
    prefetch_tmap(&tmap_w3);
    for (int i = 0; i < outm.nparts; ++i) prefetch_tmap(&outm.map[i]);
    prefetch_tmap(&outm.half);
    for (int g = 0; g < C::MAX_XG; ++g) {
      mbar_init(&x_full[g], 1);
      mbar_init(&x_empty[g], 4);
    }
    for (int s = 0; s < 2 * WP; ++s) {
      mbar_init(&w_full[s], 1);
      mbar_init(&w_empty[s], 1);
    }
    for (int kb = 0; kb < C::MAX_KB; ++kb) mbar_init(&x_ready[kb], 1);
    mbar_init(x_free, 2);  // one commit per issuer at each run boundary
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tmem_full[a], 1);
      mbar_init(&tmem_empty[a], 8);
      mbar_init(&rms_full[a], 4);
      mbar_init(&rms_empty[a], 4);
      mbar_init(&drain[a], 1);
    }
    *abort_flag = 0u;
    fence_mbarrier_init();
  }
  if (warp == C::WARP_MMA0) {
    tmem_alloc_pair(tmem_slot, C::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_relaxed();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  griddep_launch_dependents();

  if (warp >= C::WARP_WLOAD0 && warp < C::WARP_WLOAD0 + 2) {
    // W loader of pipeline pp: tiles pp, pp + 2, ... into its own WP slots of
    // two k-blocks (one 3-D load where both are whole, else 2-D loads).  It
    // walks every tile; pipeline 0's loader also loads each run's x when it
    // reaches the run's first tile (one 3-D load per group of four whole
    // k-blocks).
    const int pp = static_cast<int>(warp) - C::WARP_WLOAD0;
    if (lane == 0 && u_begin < u_end) {
      uint64_t* wf = w_full + pp * WP;
      uint64_t* we = w_empty + pp * WP;
      uint8_t* wbuf = smem + C::OFF_W + pp * WP * C::WSLOT_BYTES;
      const int rk = static_cast<int>(rank);
      TsTile t;
      int u = ts_tile(p, u_begin, u_end, t);  // tile 0
      if (pp == 0) {
        const int m0 = t.mb * 2 * C::BM + rk * C::BM;
        for (int g = 0; g < n_xg; ++g) {
          if ((g + 1) * C::XG_KB <= full_kb) tma_prefetch_3d(&tmap_x3, 0, m0, g * C::XG_KB);
          else
            for (int kb = g * C::XG_KB; kb < nkb && kb < (g + 1) * C::XG_KB; ++kb)
              tma_prefetch_2d(&tmap_x, kb * C::BK, m0);
        }
      } else if (u < u_end) {
        ts_tile(p, u, u_end, t);  // tile 1
      }
      if (pp == 0 || u < u_end) {
        const int n0 = t.n0 + rk * (t.width / 2);
        for (int s = 0; s < n_ws && s < WP; ++s) {
          if ((s + 1) * C::WS_KB <= full_kb) tma_prefetch_3d(&tmap_w3, 0, n0, s * C::WS_KB);
          else
            for (int kb = s * C::WS_KB; kb < nkb && kb < (s + 1) * C::WS_KB; ++kb)
              tma_prefetch_2d(&tmap_w, kb * C::BK, n0);
        }
      }
      griddep_wait();
      const bool arms = rank == 0;
      uint32_t stage = 0, phase = 0, xph = 0;
      int x_mb = -1;
      bool ok = true;
      for (int j = 0, uu = u_begin; uu < u_end && ok; ++j) {
        uu = ts_tile(p, uu, u_end, t);
        if (pp == 0 && t.mb != x_mb) {
          // Every x group is free again once the movers have emptied it,
          // which they do at the start of the previous run.
          x_mb = t.mb;
          const int m0 = t.mb * 2 * C::BM + rk * C::BM;
          for (int g = 0; g < n_xg && ok; ++g) {
            if (!mbar_wait(&x_empty[g], xph ^ 1u, abort_flag, to)) { ok = false; break; }
            const int kb0 = g * C::XG_KB;
            const int kbn = min(nkb, kb0 + C::XG_KB) - kb0;
            const uint32_t leader_xfull = mapa_shared(smem_addr(&x_full[g]), 0);
            if (arms)
              mbar_arrive_expect_tx(&x_full[g], static_cast<uint32_t>(2 * kbn * C::A_BYTES));
            uint8_t* dst = smem + C::OFF_X + kb0 * C::A_BYTES;
            if (kb0 + C::XG_KB <= full_kb) {
              tma_load_3d_pair(dst, &tmap_x3, leader_xfull, 0, m0, kb0);
            } else {
              for (int i = 0; i < kbn; ++i)
                tma_load_2d_pair(dst + i * C::A_BYTES, &tmap_x, leader_xfull, (kb0 + i) * C::BK,
                                 m0);
            }
          }
          xph ^= 1u;
          if (!ok) break;
        }
        if ((j & 1) != pp) continue;
        const int n0 = t.n0 + rk * (t.width / 2);
        for (int s = 0; s < n_ws; ++s) {
          if (!mbar_wait(&we[stage], phase ^ 1u, abort_flag, to)) { ok = false; break; }
          const int kb0 = s * C::WS_KB;
          const int kbn = min(nkb, kb0 + C::WS_KB) - kb0;
          const uint32_t leader_full = mapa_shared(smem_addr(&wf[stage]), 0);
          if (arms) mbar_arrive_expect_tx(&wf[stage], static_cast<uint32_t>(2 * kbn * C::B_BYTES));
          uint8_t* dst = wbuf + stage * C::WSLOT_BYTES;
          if (kb0 + C::WS_KB <= full_kb) {
            tma_load_3d_pair(dst, &tmap_w3, leader_full, 0, n0, kb0);
          } else {
            for (int i = 0; i < kbn; ++i)
              tma_load_2d_pair(dst + i * C::B_BYTES, &tmap_w, leader_full, (kb0 + i) * C::BK, n0);
          }
          if (++stage == WP) { stage = 0; phase ^= 1u; }
        }
      }
      // The MMA frees slots with a commit multicast to both CTAs: wait for the
      // last one on each slot so none lands after exit.
      for (int i = 0; i < WP && ok; ++i) {
        if (!mbar_wait(&we[stage], phase ^ 1u, abort_flag, to)) break;
        if (++stage == WP) { stage = 0; phase ^= 1u; }
      }
    }
  } else if (warp == C::WARP_MMA0 || warp == C::WARP_MMA1) {
    // MMA issuer of pipeline pp: tiles j with j % 2 == pp into accumulator pp.
    // It walks every tile to follow the runs and commits `x_free` at each run
    // boundary after its own MMAs of that run.  Pipeline 0's issuer copies
    // each run's x into TMEM at the run's first tile; its own MMAs follow the
    // copies in issue order.  Pipeline 1's issuer waits for `x_ready[kb]` on
    // its first tile of a run, and observes every phase of it in order -- a
    // run in which it has no tile is waited out at the boundary -- because a
    // parity wait cannot tell phase g from phase g - 2.
    const int pp = warp == C::WARP_MMA0 ? 0 : 1;
    if (rank == 0 && lane == 0) {
      uint64_t* wf = w_full + pp * WP;
      uint64_t* we = w_empty + pp * WP;
      const uint32_t wbuf = smem_addr(smem + C::OFF_W + pp * WP * C::WSLOT_BYTES);
      const uint32_t idesc0 = make_idesc_f16(Elem16<T>::kUmmaFormat, 2 * C::BM, 0);
      const uint32_t d_tmem = tmem_base + C::ACC_COL0 + pp * C::BN;
      uint32_t stage = 0, phase = 0;
      int j = 0, n_mine = 0, gen = -1, cur_mb = -1, mine_gen = -1;  // mine_gen: x_ready seen
      bool ok = true;
      TsTile t;
      for (int u = u_begin; u < u_end && ok; ++j) {
        u = ts_tile(p, u, u_end, t);
        if (t.mb != cur_mb) {
          ++gen;
          cur_mb = t.mb;
          if (pp == 0) {
            // Copy the run's x into TMEM columns [0, 32 * nkb).
            const uint32_t g32 = static_cast<uint32_t>(gen);
            if (gen > 0) {
              if (!mbar_wait(x_free, (g32 - 1) & 1u, abort_flag, to)) break;
              tc_fence_after();
            }
            for (int g = 0; g < n_xg && ok; ++g) {
              if (!mbar_wait(&x_full[g], g32 & 1u, abort_flag, to)) { ok = false; break; }
              tc_fence_after();
              for (int kb = g * C::XG_KB; kb < nkb && kb < (g + 1) * C::XG_KB; ++kb) {
                const uint32_t xa = smem_addr(smem + C::OFF_X + kb * C::A_BYTES);
#pragma unroll
                for (int k = 0; k < C::BK / 16; ++k)
                  tmem_cp_pair_128x256b(tmem_base + kb * 32 + k * 8,
                                        make_smem_desc_k_sw128(xa + k * 32));
                umma_commit_pair_mc(&x_ready[kb], 0x3);
              }
            }
            if (!ok) break;
            mine_gen = gen;
          }
        }
        const bool run_follows = u < u_end && u / p.units_per_mb != t.mb;
        if ((j & 1) == pp) {
          const bool first = pp == 1 && mine_gen != gen;  // pipeline 1's first tile of the run
          mine_gen = gen;
          const uint32_t acc_phase = static_cast<uint32_t>(n_mine) & 1u;
          ++n_mine;
          if (!mbar_wait_cluster(&tmem_empty[pp], acc_phase ^ 1u, abort_flag, to)) break;
          tc_fence_after();
          const uint32_t idesc = idesc0 | ((static_cast<uint32_t>(t.width) >> 3) << 17);
          for (int s = 0; s < n_ws && ok; ++s) {
            if (!mbar_wait(&wf[stage], phase, abort_flag, to)) { ok = false; break; }
            for (int i = 0; i < C::WS_KB; ++i) {
              const int kb = s * C::WS_KB + i;
              if (kb >= nkb) break;
              if (first && !mbar_wait_cluster(&x_ready[kb], static_cast<uint32_t>(gen) & 1u,
                                              abort_flag, to)) {
                ok = false;
                break;
              }
              tc_fence_after();
              const uint32_t b_addr = wbuf + stage * C::WSLOT_BYTES + i * C::B_BYTES;
#pragma unroll
              for (int k = 0; k < C::BK / 16; ++k)
                umma_f16_ts_pair(d_tmem, tmem_base + kb * 32 + k * 8,
                                 make_smem_desc_k_sw128(b_addr + k * 32), idesc,
                                 (kb > 0 || k > 0) ? 1u : 0u);
            }
            if (!ok) break;
            umma_commit_pair_mc(&we[stage], 0x3);
            if (++stage == WP) { stage = 0; phase ^= 1u; }
          }
          if (!ok) break;
          umma_commit_pair_mc(&tmem_full[pp], 0x3);
        }
        if (run_follows) {
          if (mine_gen != gen) {
            for (int kb = 0; kb < nkb && ok; ++kb)
              ok = mbar_wait_cluster(&x_ready[kb], static_cast<uint32_t>(gen) & 1u, abort_flag,
                                     to);
            mine_gen = gen;
            if (!ok) break;
          }
          umma_commit_pair_mc(x_free, 0x1);
        }
      }
      umma_commit_pair_mc(&drain[pp], 0x1);
      uint32_t zero = 0;
      mbar_wait(&drain[pp], 0, &zero, to);
    }
  } else if (warp >= C::WARP_RMS0) {
    // RMS: thread t sums x[row t]^2 over this CTA's smem copy of each run's x
    // once the k-block is in TMEM (so the copy no longer needs the smem).
    const int r = static_cast<int>((warp - C::WARP_RMS0) * 32 + lane);
    const float inv_k = 1.0f / static_cast<float>(p.K);
    int gen = -1, cur_mb = -1;
    TsTile t;
    for (int u = u_begin; u < u_end;) {
      u = ts_tile(p, u, u_end, t);
      if (t.mb == cur_mb) continue;
      cur_mb = t.mb;
      ++gen;
      const uint32_t xph = static_cast<uint32_t>(gen) & 1u;
      float ss0 = 0.f, ss1 = 0.f;
      bool ok = true;
      for (int kb = 0; kb < nkb; ++kb) {
        if (!mbar_wait(&x_ready[kb], xph, abort_flag, to)) { ok = false; break; }
        const uint32_t row = smem_addr(smem + C::OFF_X + kb * C::A_BYTES) + r * 128;
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {
          const uint4 c = ld_shared_v4(row + ((jj ^ (r & 7)) << 4));
          const float2 f0 = pair_to_float2<T>(c.x), f1 = pair_to_float2<T>(c.y);
          const float2 f2 = pair_to_float2<T>(c.z), f3 = pair_to_float2<T>(c.w);
          ss0 = fmaf(f0.x, f0.x, ss0); ss1 = fmaf(f0.y, f0.y, ss1);
          ss0 = fmaf(f1.x, f1.x, ss0); ss1 = fmaf(f1.y, f1.y, ss1);
          ss0 = fmaf(f2.x, f2.x, ss0); ss1 = fmaf(f2.y, f2.y, ss1);
          ss0 = fmaf(f3.x, f3.x, ss0); ss1 = fmaf(f3.y, f3.y, ss1);
        }
        if (kb % C::XG_KB == C::XG_KB - 1 || kb == nkb - 1) {
          __syncwarp();
          if (lane == 0) mbar_arrive(&x_empty[kb / C::XG_KB]);
        }
      }
      if (!ok) break;
      const uint32_t g2 = static_cast<uint32_t>(gen);
      if (!mbar_wait(&rms_empty[g2 & 1], ((g2 >> 1) & 1) ^ 1u, abort_flag, to)) break;
      rms_buf[(g2 & 1) * C::BM + r] = rsqrtf((ss0 + ss1) * inv_k + p.eps);
      __syncwarp();
      if (lane == 0) mbar_arrive(&rms_full[g2 & 1]);
    }
  } else {
    // Epilogue: warp q owns TMEM lanes [32q, 32q+32) = rows of this CTA's
    // half; tile j sits in accumulator j % 2.
    const uint32_t q = warp;
    const T* bias = static_cast<const T*>(p.bias);
    const uint32_t leader_tmem_empty0 = mapa_shared(smem_addr(&tmem_empty[0]), 0);
    int ntiles = 0;
    {
      TsTile t;
      for (int u = u_begin; u < u_end; ++ntiles) u = ts_tile(p, u, u_end, t);
    }
    griddep_wait();
    uint32_t nst = 0;  // chunks this warp has staged: staging buffer nst & 1
    int j = 0, gen = -1, cur_mb = -1;
    float inv_rms = 0.f;
    TsTile t;
    for (int u = u_begin; u < u_end; ++j) {
      u = ts_tile(p, u, u_end, t);
      const bool first = t.mb != cur_mb;
      if (first) { ++gen; cur_mb = t.mb; }
      const bool last = u >= u_end || u / p.units_per_mb != t.mb;
      const uint32_t g = static_cast<uint32_t>(gen);
      const uint32_t acc = j & 1, acc_phase = (j >> 1) & 1;
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
      const int row_base = t.mb * 2 * C::BM + static_cast<int>(rank) * C::BM + q * 32;
      ts_epilogue_tile<T>(smem + C::OFF_STG + q * 2 * C::STG_BYTES, lane,
                          tmem_base + C::ACC_COL0 + acc * C::BN + ((q * 32u) << 16), t.n0,
                          row_base, inv_rms, bias, p.N, outm, nst, j + 2 < ntiles,
                          leader_tmem_empty0 + acc * 8, t.width);
    }
    if (lane == 0) bulk_wait_group_read<0>();
  }

  __syncwarp();
  tc_fence_before();
  cluster_sync_relaxed();
  if (*abort_flag) __nanosleep(20000);
  if (warp == C::WARP_MMA0) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
  }
}

// ------------------------------------------------------------------ host side

// Unit ranges per pair.  When every m-block can have pairs of its own, the
// pairs are dealt out to m-blocks (so no pair loads x twice) and each
// m-block's units split evenly among its pairs; otherwise the m-block-major
// unit sequence is cut into equal contiguous ranges (a range that crosses an
// m-block reloads x once).  The first choice is taken unless its busiest
// pair carries more than one unit above the second's.
static int ts_schedule(int64_t num_mb, int64_t upm, int pairs_avail, TsSchedule* s) {
  const int64_t total = num_mb * upm;
  int pairs = pairs_avail < kTsMaxPairs ? pairs_avail : kTsMaxPairs;
  if (total < pairs) pairs = static_cast<int>(total);
  const int64_t max_contig = (total + pairs - 1) / pairs;
  bool aligned = false;
  if (num_mb <= pairs) {
    const int64_t min_pairs_per_mb = pairs / num_mb;
    const int64_t max_aligned = (upm + min_pairs_per_mb - 1) / min_pairs_per_mb;
    aligned = max_aligned <= max_contig + 1;
  }
  if (aligned) {
    int idx = 0;
    for (int64_t b = 0; b < num_mb; ++b) {
      const int64_t pb = pairs / num_mb + (b < pairs % num_mb ? 1 : 0);
      for (int64_t j = 0; j < pb; ++j) s->u0[idx++] = static_cast<int32_t>(b * upm + j * upm / pb);
    }
  } else {
    for (int i = 0; i < pairs; ++i) s->u0[i] = static_cast<int32_t>(total * i / pairs);
  }
  s->u0[pairs] = static_cast<int32_t>(total);
  return pairs;
}

template <typename T, int WP>
static int launch_ts(const LinearProblem& pr, cudaStream_t stream) {
  using C = TsCfg<WP>;
  auto kern = fused_rmsnorm_linear_ts_kernel<T, WP>;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return set_cuda_error("cudaGetDevice");
  static int max_pairs[kMaxDevices] = {};
  if (dev < kMaxDevices && max_pairs[dev] == 0) {
    cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
    if (e != cudaSuccess) return set_cuda_error("cudaFuncSetAttribute(ts kernel)", e);
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
  if (pr.K > C::MAX_KB * C::BK)
    return set_error(FRN_ERR_UNSUPPORTED, "the x-in-TMEM kernel takes K <= %d (got %lld)",
                     C::MAX_KB * C::BK, (long long)pr.K);
  const bool split = pr.parts && pr.parts->n > 1;
  const CUtensorMapDataType dt = Elem16<T>::kTmaType;
  CUtensorMap tx, tw, tx3, tw3;
  int rc = encode_tmap_2d(&tx, dt, 2, pr.x, pr.K, pr.M, pr.x_row_stride, C::BK, C::BM,
                          CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = encode_tmap_2d(&tw, dt, 2, pr.w, pr.K, pr.N, pr.w_row_stride, C::BK, C::BN_HALF,
                      CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  // 3-D k-block views (x: 4 k-blocks per load, W: 2); used only where every
  // k-block of a load is whole.
  if (pr.K >= C::BK) {
    rc = encode_tmap_kblocks_3d(&tx3, dt, pr.x, pr.K, pr.M, pr.x_row_stride, C::BM, C::XG_KB);
    if (rc) return rc;
    rc = encode_tmap_kblocks_3d(&tw3, dt, pr.w, pr.K, pr.N, pr.w_row_stride, C::BN_HALF,
                                C::WS_KB);
    if (rc) return rc;
  } else {
    tx3 = tx;
    tw3 = tw;
  }
  PairOut outm;
  rc = build_pair_out(pr, pr.N, !split, &outm);
  if (rc) return rc;

  TsParams p;
  p.M = static_cast<int32_t>(pr.M);
  p.N = static_cast<int32_t>(pr.N);
  p.K = static_cast<int32_t>(pr.K);
  p.num_k_blocks = static_cast<int32_t>((pr.K + C::BK - 1) / C::BK);
  p.unit_cols = split ? 64 : 32;
  p.tile_units = C::BN / p.unit_cols;
  p.units_per_mb = static_cast<int32_t>((pr.N + p.unit_cols - 1) / p.unit_cols);
  p.eps = pr.eps;
  p.bias = pr.bias;
  p.timeout_ns = wait_timeout_ns();
  const int64_t num_mb = (pr.M + 2 * C::BM - 1) / (2 * C::BM);
  if (num_mb * p.units_per_mb > INT32_MAX)
    return set_error(FRN_ERR_UNSUPPORTED, "problem too large for the x-in-TMEM kernel");
  TsSchedule sched;
  const int pairs = ts_schedule(num_mb, p.units_per_mb, pairs_avail, &sched);

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
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, tx, tx3, tw, tw3, outm, sched, p);
  if (e != cudaSuccess) return set_cuda_error("launch fused_rmsnorm_linear_ts", e);
  return 0;
}

int run_fused_linear_ts(const LinearProblem& pr, cudaStream_t s) {
  if (pr.dtype == FRN_DTYPE_BF16) return launch_ts<__nv_bfloat16, 2>(pr, s);
  if (pr.dtype == FRN_DTYPE_F16) return launch_ts<__half, 2>(pr, s);
  return set_error(FRN_ERR_UNSUPPORTED, "fused RMSNorm+Linear supports bf16 and fp16 only");
}

}  // namespace frn
