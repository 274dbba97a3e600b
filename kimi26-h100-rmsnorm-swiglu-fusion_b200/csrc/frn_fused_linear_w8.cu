// frn_fused_linear_w8.cu -- fused RMSNorm -> Linear with int8 weights.
//
//   out[m, n] = round(inv_rms[m] * scale[n] * sum_k x[m,k] * q[n,k] + b[n])
//
// q is the gamma-folded weight quantized per output channel (symmetric,
// scale[n] = max|W_fused[n,:]| / 127, q = clamp(round(W_fused / scale), +-127);
// the quantizer of the reference's quantization-aware benchmark,
// src/benchmark_kimi26_quantized.py:30-35).  Where the reference dequantizes
// the whole weight to bf16 in HBM on every call and then runs F.linear on
// x * bf16(inv_rms) (:38-39, :102-106), this kernel streams the int8 bytes
// (half the weight traffic of bf16) and widens them to bf16 in shared memory
// right before the tensor cores read them.  |q| <= 127 is exact in bf16, so
// the product is the exact integer dot product accumulated in fp32; inv_rms
// and scale are applied once, to the fp32 accumulator.
//
// Layout: the SM-pair (cta_group::2) kernel of frn_fused_linear_pair.cu with
// one more role and two rings.  The main ring's stage holds, per CTA, the x
// tile [128 x 64] bf16 (TMA, completes on the even CTA's `full`) and the bf16
// copy of this CTA's W half-tile, which the converter warps write in the UMMA
// 128B-swizzled K-major layout and announce on the even CTA's `conv` barrier
// (its own converter arrives and expects 4 bytes, which the odd CTA's
// converter sends with st.async).  The int8 half-tiles [BN/2 x 64] (TMA,
// 64B-swizzled) stream through a ring of their own, QST slots deep, so they
// are in shared memory well before a converter needs them: the conversion,
// not the int8 load latency, is what the main ring waits for.
//
// Roles (each CTA): warps 0-3 epilogue, warps 4 and 15 x producers (even /
// odd k-blocks of the sequence: one thread completes a tensor TMA only every
// few hundred clocks), warp 5 int8 producer, warp 6 MMA (even CTA) + TMEM
// owner, warps 7-10 RMS, warps 11-14 converters (k-block sequence mod 4,
// lane = W rows of the half-tile).
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>

#include "frn_internal.h"
#include "frn_ptx.cuh"

namespace frn {

struct W8Params {
  int32_t M, N, K;
  int32_t num_m_blocks, num_n_blocks, num_k_blocks;
  float eps;
  const float* scale;  // [N] per-output-channel dequantization scales
  const void* bias;    // may be null
  void* out;
  int64_t out_row_stride;
  uint64_t timeout_ns;
};

// One launch serves one or two independent problems (same x type and tile
// width, e.g. an MLA layer's q_b and kv_b, which read different inputs): each
// pair takes a balanced contiguous run of each problem's tiles (problem 1's
// runs in reverse pair order, so a pair with an extra problem-0 tile gets one
// fewer of problem 1), problem 0's first.  The rings, the accumulators and
// the inv_rms buffers carry on from one problem to the next, so the second
// problem's mainloop overlaps the first one's last epilogue.
struct W8Group {
  W8Params p[2];
  int32_t nprob;
};

struct W8Maps {
  CUtensorMap x[2], q[2], out[2], out_half[2];
};

// Tiles [tb, te) of problem j for pair `pair` of `npairs`.
__device__ __forceinline__ void w8_tile_range(const W8Params& q, int j, int pair, int npairs,
                                              int& tb, int& te) {
  const int tiles = q.num_m_blocks * q.num_n_blocks;
  const int pr = j == 0 ? pair : npairs - 1 - pair;
  const int base = tiles / npairs, rem = tiles % npairs;
  tb = pr * base + min(pr, rem);
  te = tb + base + (pr < rem ? 1 : 0);
}

template <int BN, int STAGES, int QST>
struct W8Cfg {
  static constexpr int BM = 128;
  static constexpr int BK = 64;
  static constexpr int BN_HALF = BN / 2;
  static constexpr int A_BYTES = BM * BK * 2;        // bf16 x tile
  static constexpr int Q_BYTES = BN_HALF * BK;        // int8 W half-tile
  static constexpr int B_BYTES = BN_HALF * BK * 2;   // its bf16 copy
  static constexpr uint32_t PAIR_A_TX = 2u * A_BYTES;
  static constexpr uint32_t TMEM_COLS = (2 * BN <= 256) ? 256u : 512u;
  static constexpr int STG_BYTES = 32 * 128;
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = OFF_A + STAGES * A_BYTES;
  static constexpr int OFF_Q = OFF_B + STAGES * B_BYTES;
  static constexpr int OFF_STG = OFF_Q + QST * Q_BYTES;
  static constexpr int OFF_RMS = OFF_STG + 4 * 2 * STG_BYTES;
  static constexpr int OFF_SCL = OFF_RMS + 2 * BM * 4;  // per epilogue warp: the tile's scale[n]
  static constexpr int OFF_BAR = OFF_SCL + 4 * BN * 4;
  static constexpr int NCHUNK = (BN + 63) / 64;  // epilogue chunks of 64 columns
  static constexpr bool HALF_TAIL = BN % 64 != 0;
  static constexpr int NUM_BARS = 4 * STAGES + 2 * QST + 9;
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
  static constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;
  static constexpr int EPI_WARPS = 4, RMS_WARPS = 4, CONV_WARPS = 4;
  static constexpr int WARP_XLOAD = 4, WARP_QLOAD = 5, WARP_MMA = 6, WARP_RMS0 = 7,
                       WARP_CONV0 = 11, WARP_XLOAD1 = 15;
  static constexpr int THREADS = 32 * 16;
  static_assert(B_BYTES % 1024 == 0 && Q_BYTES % 1024 == 0, "stage buffers must stay aligned");
  // The converter warps take the k-block sequence in turn; their parity waits
  // stay unambiguous only with rings at least as deep as the warps are many.
  static_assert(STAGES >= CONV_WARPS && QST >= CONV_WARPS, "rings shallower than the converters");
  static_assert(OFF_STG % 1024 == 0, "staging blocks must be 1024-aligned for the 128B swizzle");
  static_assert(SMEM_BYTES <= 232448, "exceeds 227 KB of dynamic shared memory");
};

// Four signed int8 (one 32-bit word, |q| <= 127) -> four exact 16-bit values
// of T as two packed pairs {q0, q1}, {q2, q3}.  No int->float converter:
//  bf16: put byte q+128 in the low mantissa bits of 2^23 and subtract 2^23 +
//        128 in fp32 (magic-number conversion, e.g. Kim et al. 2022, "Who Says
//        Elephants Can't Run"; two lanes per add.rn.f32x2), then keep the top
//        16 bits -- exact, because |q| <= 127 has at most 7 significant bits;
//  fp16: the same with 2^10 in half precision (0x6400 | (q+128)) minus 1152,
//        two lanes per sub.f16x2.
template <typename T>
__device__ __forceinline__ void widen_s8x4(uint32_t w, uint32_t& o01, uint32_t& o23);

template <>
__device__ __forceinline__ void widen_s8x4<__nv_bfloat16>(uint32_t w, uint32_t& o01,
                                                          uint32_t& o23) {
  const uint32_t u = w ^ 0x80808080u;  // q + 128 in every byte
  uint64_t p01 = (static_cast<uint64_t>(__byte_perm(u, 0x4B000000u, 0x7651)) << 32) |
                 __byte_perm(u, 0x4B000000u, 0x7650);
  uint64_t p23 = (static_cast<uint64_t>(__byte_perm(u, 0x4B000000u, 0x7653)) << 32) |
                 __byte_perm(u, 0x4B000000u, 0x7652);
  const uint64_t bias = 0xCB000080CB000080ull;  // -(2^23 + 128) in both lanes
  asm("add.rn.f32x2 %0, %0, %2;\n\tadd.rn.f32x2 %1, %1, %2;"
      : "+l"(p01), "+l"(p23)
      : "l"(bias));
  o01 = __byte_perm(static_cast<uint32_t>(p01), static_cast<uint32_t>(p01 >> 32), 0x7632);
  o23 = __byte_perm(static_cast<uint32_t>(p23), static_cast<uint32_t>(p23 >> 32), 0x7632);
}

template <>
__device__ __forceinline__ void widen_s8x4<__half>(uint32_t w, uint32_t& o01, uint32_t& o23) {
  const uint32_t u = w ^ 0x80808080u;
  const uint32_t h01 = __byte_perm(u, 0x64646464u, 0x4140);  // {1024 + u0, 1024 + u1}
  const uint32_t h23 = __byte_perm(u, 0x64646464u, 0x4342);
  const uint32_t c = 0x64806480u;                           // {1152, 1152}
  asm("sub.rn.f16x2 %0, %2, %4;\n\tsub.rn.f16x2 %1, %3, %4;"
      : "=r"(o01), "=r"(o23)
      : "r"(h01), "r"(h23), "r"(c));
}

template <typename T, int BN, int STAGES, int QST>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(W8Cfg<BN, STAGES, QST>::THREADS, 1)
    fused_rmsnorm_linear_w8_kernel(const __grid_constant__ W8Maps maps,
                                   const __grid_constant__ W8Group grp) {
  using C = W8Cfg<BN, STAGES, QST>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));

  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);  // even CTA: x of both CTAs
  uint64_t* conv = full + STAGES;                                  // even CTA: bf16 W ready
  uint64_t* mma_done = conv + STAGES;
  uint64_t* empty = mma_done + STAGES;
  uint64_t* qfull = empty + STAGES;   // [QST] this CTA's int8 tile landed
  uint64_t* qempty = qfull + QST;     // [QST] its converter is done with it
  uint64_t* tmem_full = qempty + QST;
  uint64_t* tmem_empty = tmem_full + 2;
  uint64_t* rms_full = tmem_empty + 2;
  uint64_t* rms_empty = rms_full + 2;
  uint64_t* drain = rms_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile uint32_t* abort_flag = tmem_slot + 1;
  float* rms_buf = reinterpret_cast<float*>(smem + C::OFF_RMS);

  const uint32_t warp = warp_id_in_cta();
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t rank = cluster_cta_rank();
  const uint32_t pair = blockIdx.x >> 1;
  const uint32_t num_pairs = gridDim.x >> 1;

  if (warp == C::WARP_XLOAD && lane == 0) {
    for (int j = 0; j < grp.nprob; ++j) {
      prefetch_tmap(&maps.x[j]);
      prefetch_tmap(&maps.q[j]);
      prefetch_tmap(&maps.out[j]);
      if (C::HALF_TAIL) prefetch_tmap(&maps.out_half[j]);
    }
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&conv[s], 1);  // even CTA's converter arrives; odd CTA's sends 4 tx bytes
      mbar_init(&mma_done[s], 1);
      mbar_init(&empty[s], C::RMS_WARPS);
    }
    for (int s = 0; s < QST; ++s) {
      mbar_init(&qfull[s], 1);
      mbar_init(&qempty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tmem_full[a], 1);
      mbar_init(&tmem_empty[a], 2 * C::EPI_WARPS);
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
  // This CTA's inits and TMEM slot reach its own threads through
  // __syncthreads; the peer's inits were released by its fence.mbarrier_init.
  __syncthreads();
  cluster_sync_relaxed();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // This pair's contiguous m-block-major run of each problem's tiles
  // (inv_rms once per run), and how many tiles and k-blocks that is in all.
  int tb[2] = {0, 0}, te[2] = {0, 0};
  int pair_tiles = 0, pair_kbs = 0;
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    if (j < grp.nprob) {
      w8_tile_range(grp.p[j], j, static_cast<int>(pair), static_cast<int>(num_pairs), tb[j], te[j]);
      pair_tiles += te[j] - tb[j];
      pair_kbs += (te[j] - tb[j]) * grp.p[j].num_k_blocks;
    }
  }
  const int j0 = te[0] > tb[0] ? 0 : 1;  // the problem of this pair's first tile
  const int tb_first = j0 == 0 ? tb[0] : tb[1], te_first = j0 == 0 ? te[0] : te[1];
  const uint64_t to = grp.p[0].timeout_ns;
  // Let the next kernel in the stream get scheduled now: its CTAs take SMs as
  // ours retire and run their set-up while we finish; its griddepcontrol.wait
  // still orders all of its global accesses after this whole grid.
  griddep_launch_dependents();

  if (warp == C::WARP_XLOAD || warp == C::WARP_XLOAD1) {
    // x tiles into the main ring (both CTAs' halves complete on the even
    // CTA's `full`, armed by the even CTA); this thread takes the k-blocks
    // of the sequence with i % 2 == sel.
    if (lane == 0) {
      const uint32_t sel = warp == C::WARP_XLOAD ? 0u : 1u;
      // While the preceding grid drains, pull this thread's share of the first
      // ring of x tiles into L2.
      if (tb_first < te_first) {
        const W8Params& pf = grp.p[j0];
        const int pm0 = (tb_first / pf.num_n_blocks) * 2 * C::BM + rank * C::BM;
        for (int kb = static_cast<int>(sel); kb < pf.num_k_blocks && kb < STAGES; kb += 2)
          tma_prefetch_2d(&maps.x[j0], kb * C::BK, pm0);
      }
      griddep_wait();
      uint32_t i = 0;
      bool ok = true;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const W8Params& pj = grp.p[j];
        for (int t = tb[j]; t < te[j] && ok; ++t) {
          const int m0 = (t / pj.num_n_blocks) * 2 * C::BM + rank * C::BM;
          for (int kb = 0; kb < pj.num_k_blocks; ++kb, ++i) {
            if ((i & 1u) != sel) continue;
            const uint32_t s = i % STAGES, ph = (i / STAGES) & 1u;
            if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, to)) { ok = false; break; }
            const uint32_t leader_full = mapa_shared(smem_addr(&full[s]), 0);
            if (rank == 0) mbar_arrive_expect_tx(&full[s], C::PAIR_A_TX);
            tma_load_2d_pair(smem + C::OFF_A + s * C::A_BYTES, &maps.x[j], leader_full,
                             kb * C::BK, m0);
          }
        }
      }
    }
  } else if (warp == C::WARP_QLOAD) {
    // int8 half-tiles into their own ring, as far ahead as its QST slots go.
    if (lane == 0) {
      if (tb_first < te_first) {  // the first ring of int8 tiles into L2 likewise
        const W8Params& pf = grp.p[j0];
        const int pn0 = (tb_first % pf.num_n_blocks) * BN + rank * C::BN_HALF;
        for (int kb = 0; kb < pf.num_k_blocks && kb < QST; ++kb)
          tma_prefetch_2d(&maps.q[j0], kb * C::BK, pn0);
      }
      griddep_wait();
      uint32_t i = 0;
      bool ok = true;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const W8Params& pj = grp.p[j];
        for (int t = tb[j]; t < te[j] && ok; ++t) {
          const int n0 = (t % pj.num_n_blocks) * BN + rank * C::BN_HALF;
          for (int kb = 0; kb < pj.num_k_blocks; ++kb, ++i) {
            const uint32_t qs = i % QST, qph = (i / QST) & 1u;
            if (!mbar_wait(&qempty[qs], qph ^ 1u, abort_flag, to)) { ok = false; break; }
            mbar_arrive_expect_tx(&qfull[qs], C::Q_BYTES);
            tma_load_2d(smem + C::OFF_Q + qs * C::Q_BYTES, &maps.q[j], &qfull[qs], kb * C::BK,
                        n0);
          }
        }
      }
    }
  } else if (warp == C::WARP_MMA) {
    if (rank == 0 && lane == 0) {
      const uint32_t idesc = make_idesc_f16(Elem16<T>::kUmmaFormat, 2 * C::BM, BN);
      uint32_t stage = 0, phase = 0;
      int i = 0;
      bool ok = true;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int nkb = grp.p[j].num_k_blocks;
        for (int t = tb[j]; t < te[j] && ok; ++t, ++i) {
          const uint32_t acc = i & 1, acc_phase = (i >> 1) & 1;
          if (!mbar_wait_cluster(&tmem_empty[acc], acc_phase ^ 1u, abort_flag, to)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + acc * BN;
          for (int kb = 0; kb < nkb; ++kb) {
            if (!mbar_wait(&full[stage], phase, abort_flag, to)) { ok = false; break; }
            // As for the pair's TMA loads (data in the odd CTA, complete_tx on this
            // barrier), a CTA-scope wait suffices: the odd CTA's half arrives as
            // an st.async complete_tx, itself ordered after that CTA's
            // fence.proxy.async.  (A cluster-scope acquire here cost ~0.25 us
            // per k-block on the critical path.)
            if (!mbar_wait(&conv[stage], phase, abort_flag, to)) { ok = false; break; }
            tc_fence_after();
            const uint32_t a_addr = smem_addr(smem + C::OFF_A + stage * C::A_BYTES);
            const uint32_t b_addr = smem_addr(smem + C::OFF_B + stage * C::B_BYTES);
#pragma unroll
            for (int k = 0; k < C::BK / 16; ++k)
              umma_f16_ss_pair(d_tmem, make_smem_desc_k_sw128(a_addr + k * 32),
                               make_smem_desc_k_sw128(b_addr + k * 32), idesc,
                               (kb > 0 || k > 0) ? 1u : 0u);
            umma_commit_pair_mc(&mma_done[stage], 0x3);
            if (++stage == STAGES) { stage = 0; phase ^= 1u; }
          }
          if (!ok) break;
          umma_commit_pair_mc(&tmem_full[acc], 0x3);
        }
      }
      umma_commit_pair_mc(drain, 0x1);
      uint32_t zero = 0;
      mbar_wait(drain, 0, &zero, to);
    }
  } else if (warp >= C::WARP_CONV0) {
    // Converter warp cw widens every CONV_WARPS-th k-block of the sequence
    // (up to CONV_WARPS stages convert at once, for any ring depth): lane l
    // takes rows l, l+32, ... of this CTA's int8 half-tile, then lane 0
    // publishes the stage on the even CTA's `conv` barrier.
    const uint32_t cw = warp - C::WARP_CONV0;
    const uint32_t leader_conv0 = mapa_shared(smem_addr(&conv[0]), 0);
    const uint32_t leader_sink = mapa_shared(smem_addr(tmem_slot + 2), 0);
    const uint32_t q0 = smem_addr(smem + C::OFF_Q), b0 = smem_addr(smem + C::OFF_B);
    const uint32_t total = static_cast<uint32_t>(pair_kbs);
    for (uint32_t i = cw; i < total; i += C::CONV_WARPS) {
      const uint32_t qs = i % QST, qph = (i / QST) & 1u;
      const uint32_t stage = i % STAGES, phase = (i / STAGES) & 1u;
      // The slot's previous tile (use i - QST, another warp's) has been
      // released first: only then is qfull[qs] in this use's phase.  A wait on
      // the parity alone could match that previous phase while it is still
      // pending (its tile landing after the ones this warp just converted)
      // and convert a tile that has not arrived.  (The release wait itself
      // cannot alias: the loader had to see use i - 2*QST released before it
      // issued use i - 4, which this warp converted, and QST >= 4.)
      if (!mbar_wait(&qempty[qs], qph ^ 1u, abort_flag, to)) break;
      // The int8 tile has landed, and the main slot's previous MMA is done
      // (its RMS warps released it).
      if (!mbar_wait(&qfull[qs], qph, abort_flag, to)) break;
      if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, to)) break;
      const uint32_t qsa = q0 + qs * C::Q_BYTES, bs = b0 + stage * C::B_BYTES;
#pragma unroll 2
      for (uint32_t j = lane; j < static_cast<uint32_t>(C::BN_HALF); j += 32) {
        // int8 row j: 64 bytes, 64B-swizzled (16-byte chunk c at c ^ ((j >> 1) & 3));
        // bf16 row j: 128 bytes, 128B-swizzled (chunk c at c ^ (j & 7)).
        uint4 w[4];
#pragma unroll
        for (uint32_t c = 0; c < 4; ++c)
          w[c] = ld_shared_v4(qsa + j * 64 + ((c ^ ((j >> 1) & 3u)) << 4));
#pragma unroll
        for (uint32_t c = 0; c < 4; ++c) {
          uint32_t o[8];
          widen_s8x4<T>(w[c].x, o[0], o[1]);
          widen_s8x4<T>(w[c].y, o[2], o[3]);
          widen_s8x4<T>(w[c].z, o[4], o[5]);
          widen_s8x4<T>(w[c].w, o[6], o[7]);
          st_shared_v4(bs + j * 128 + (((2 * c) ^ (j & 7u)) << 4), o[0], o[1], o[2], o[3]);
          st_shared_v4(bs + j * 128 + (((2 * c + 1) ^ (j & 7u)) << 4), o[4], o[5], o[6], o[7]);
        }
      }
      // The tensor cores (async proxy) read what was just written.  The even
      // CTA arrives locally and expects 4 bytes; the odd CTA sends them with
      // st.async, whose complete_tx on the even CTA's barrier is a
      // cluster-scope release that does not stall this warp (a releasing
      // remote arrive costs a few hundred cycles here).
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&qempty[qs]);
        if (rank == 0)
          mbar_arrive_expect_tx(&conv[stage], 4u);
        else
          st_async_complete_tx(leader_sink, 1u, leader_conv0 + stage * 8);
      }
    }
  } else if (warp >= C::WARP_RMS0) {
    const int r = static_cast<int>(threadIdx.x) - C::WARP_RMS0 * 32;
    uint32_t stage = 0, phase = 0;
    int gen = -1;
    bool ok = true;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const W8Params& pj = grp.p[j];
      int cur_m = -1;
      for (int t = tb[j]; t < te[j] && ok; ++t) {
        const int mb = t / pj.num_n_blocks;
        const bool first = (mb != cur_m);
        if (first) { ++gen; cur_m = mb; }
        float ss0 = 0.f, ss1 = 0.f;
        for (int kb = 0; kb < pj.num_k_blocks; ++kb) {
          if (!mbar_wait(&mma_done[stage], phase, abort_flag, to)) { ok = false; break; }
          if (first) {
            const uint32_t row = smem_addr(smem + C::OFF_A + stage * C::A_BYTES) + r * 128;
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
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
        if (!ok || !first) continue;
        const uint32_t g = static_cast<uint32_t>(gen);
        if (!mbar_wait(&rms_empty[g & 1], ((g >> 1) & 1) ^ 1u, abort_flag, to)) {
          ok = false;
          break;
        }
        const float inv_k = 1.0f / static_cast<float>(pj.K);
        rms_buf[(g & 1) * C::BM + r] = rsqrtf((ss0 + ss1) * inv_k + pj.eps);
        __syncwarp();
        if (lane == 0) mbar_arrive(&rms_full[g & 1]);
      }
    }
  } else {
    // Epilogue warps 0-3 (as in the bf16 pair kernel, plus scale[n]).
    const uint32_t q = warp;
    const uint32_t leader_tmem_empty0 = mapa_shared(smem_addr(&tmem_empty[0]), 0);
    const uint32_t scl = smem_addr(smem + C::OFF_SCL + q * BN * 4);  // this warp's scale[n0 ..)
    griddep_wait();
    uint32_t nst = 0;  // chunks this warp has staged: staging buffer nst & 1
    int i = 0;
    int gen = -1;
    float inv_rms = 0.f;
    bool ok = true;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const W8Params& pj = grp.p[j];
      int cur_m = -1;
      for (int t = tb[j]; t < te[j] && ok; ++t, ++i) {
        const bool has_bias = pj.bias != nullptr;
        const T* bias = static_cast<const T*>(pj.bias);
        const uint32_t acc = i & 1, acc_phase = (i >> 1) & 1;
        const int mb = t / pj.num_n_blocks;
        const int row_base = mb * 2 * C::BM + rank * C::BM + q * 32;
        const int n0 = (t % pj.num_n_blocks) * BN;
        const bool first = (mb != cur_m);
        const bool last = (t + 1 >= te[j]) || ((t + 1) / pj.num_n_blocks != mb);
        const bool reuse_acc = i + 2 < pair_tiles;  // a later tile (of either problem) uses acc
        if (first) { ++gen; cur_m = mb; }
        const uint32_t g = static_cast<uint32_t>(gen);
        // The tile's column scales (0 past N) into this warp's slice; N % 8 == 0,
        // so a group of 4 columns is either wholly inside or wholly past N.
        for (int c4 = static_cast<int>(lane); c4 < BN / 4; c4 += 32) {
          const int col = n0 + c4 * 4;
          uint4 sv = make_uint4(0u, 0u, 0u, 0u);
          if (col < pj.N) sv = ld_global_nc_v4(pj.scale + col);
          st_shared_v4(scl + c4 * 16, sv.x, sv.y, sv.z, sv.w);
        }
        __syncwarp();
        if (!mbar_wait(&tmem_full[acc], acc_phase, abort_flag, to)) {
          ok = false;
          break;
        }
        if (first) {
          if (!mbar_wait(&rms_full[g & 1], (g >> 1) & 1, abort_flag, to)) {
            ok = false;
            break;
          }
          inv_rms = rms_buf[(g & 1) * C::BM + q * 32 + lane];
        }
        tc_fence_after();
        if (last) {
          __syncwarp();
          if (lane == 0) mbar_arrive(&rms_empty[g & 1]);
        }
        const uint32_t taddr = tmem_base + acc * BN + ((q * 32u) << 16);
#pragma unroll 1
        for (int c = 0; c < C::NCHUNK; ++c, ++nst) {
          const bool half = C::HALF_TAIL && c == C::NCHUNK - 1;
          const int col0 = n0 + c * 64;
          uint4 bv[8];
          if (has_bias) {
#pragma unroll
            for (int c8 = 0; c8 < 8; ++c8)
              bv[c8] = (col0 + c8 * 8 < pj.N && !(half && c8 >= 4))
                           ? ld_global_nc_v4(bias + col0 + c8 * 8)
                           : make_uint4(0u, 0u, 0u, 0u);
          }
          uint32_t v[64];
          tmem_ld_32x32b_x32(taddr + c * 64, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
          if (!half)
            tmem_ld_32x32b_x32(taddr + c * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
          tmem_ld_wait();
          if (c == C::NCHUNK - 1 && reuse_acc) {
            // Only a later tile of this pair waits for this accumulator.
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster_relaxed(leader_tmem_empty0 + acc * 8);
          }
          uint8_t* sbp = smem + C::OFF_STG + (q * 2 + (nst & 1u)) * C::STG_BYTES;
          const uint32_t sb = smem_addr(sbp);
          if (lane == 0) bulk_wait_group_read<1>();
          __syncwarp();
          const uint32_t cs = scl + c * 64 * 4;
          if (half) {
            if (has_bias) stage_rows_swizzled<T, 4, true, true>(v, inv_rms, bv, sb, lane, cs);
            else stage_rows_swizzled<T, 4, false, true>(v, inv_rms, bv, sb, lane, cs);
          } else {
            if (has_bias) stage_rows_swizzled<T, 8, true, true>(v, inv_rms, bv, sb, lane, cs);
            else stage_rows_swizzled<T, 8, false, true>(v, inv_rms, bv, sb, lane, cs);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(half ? &maps.out_half[j] : &maps.out[j], sbp, col0, row_base);
            bulk_commit_group();
          }
        }
      }
    }
    if (lane == 0) bulk_wait_group_read<0>();
  }

  // Every cross-CTA signal has been waited for by its target by now.
  __syncwarp();
  tc_fence_before();
  cluster_sync_relaxed();
  if (*abort_flag) __nanosleep(20000);
  if (warp == C::WARP_MMA) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
  }
}

// ------------------------------------------------------------------ quantizer

// Symmetric per-output-channel int8 quantization of the folded weight, one CTA
// per row: scale = max(|w|, 1e-8) / 127 in fp32, q = clamp(rint(w / scale),
// -127, 127) -- round half to even, IEEE division, exactly torch.round(w /
// scale).clamp(-127, 127) of the reference (src/benchmark_kimi26_quantized.py:30-35).
template <typename T>
__global__ void __launch_bounds__(256) quantize_rows_kernel(const T* __restrict__ w, int64_t ws,
                                                            int K, int8_t* __restrict__ q,
                                                            int64_t qs, float* __restrict__ scale) {
  __shared__ float red[8];
  const T* row = w + static_cast<int64_t>(blockIdx.x) * ws;
  float amax = 0.f;
  for (int k = threadIdx.x; k < K; k += 256) amax = fmaxf(amax, fabsf(static_cast<float>(row[k])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  float m = red[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) m = fmaxf(m, red[i]);
  const float sc = fmaxf(m, 1e-8f) / 127.0f;
  if (threadIdx.x == 0) scale[blockIdx.x] = sc;
  int8_t* qrow = q + static_cast<int64_t>(blockIdx.x) * qs;
  for (int k = threadIdx.x; k < K; k += 256) {
    float v = rintf(static_cast<float>(row[k]) / sc);
    v = fminf(fmaxf(v, -127.f), 127.f);
    qrow[k] = static_cast<int8_t>(v);
  }
}

int run_quantize_int8(int dtype, const void* w, int64_t N, int64_t K, int64_t ws, void* q,
                      int64_t qs, float* scale, cudaStream_t s) {
  if (dtype == FRN_DTYPE_BF16)
    quantize_rows_kernel<__nv_bfloat16><<<static_cast<unsigned>(N), 256, 0, s>>>(
        static_cast<const __nv_bfloat16*>(w), ws, static_cast<int>(K), static_cast<int8_t*>(q), qs,
        scale);
  else if (dtype == FRN_DTYPE_F16)
    quantize_rows_kernel<__half><<<static_cast<unsigned>(N), 256, 0, s>>>(
        static_cast<const __half*>(w), ws, static_cast<int>(K), static_cast<int8_t*>(q), qs, scale);
  else if (dtype == FRN_DTYPE_F32)
    quantize_rows_kernel<float><<<static_cast<unsigned>(N), 256, 0, s>>>(
        static_cast<const float*>(w), ws, static_cast<int>(K), static_cast<int8_t*>(q), qs, scale);
  else
    return set_error(FRN_ERR_UNSUPPORTED, "quantize: weight dtype must be fp32, fp16 or bf16");
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error("launch quantize_rows", e);
  return 0;
}

// ------------------------------------------------------------------ host side

template <typename T, int BN, int STAGES, int QST>
static int launch_w8(const W8Problem* prs, int nprob, cudaStream_t stream) {
  using C = W8Cfg<BN, STAGES, QST>;
  auto kern = fused_rmsnorm_linear_w8_kernel<T, BN, STAGES, QST>;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return set_cuda_error("cudaGetDevice");
  static int max_pairs[kMaxDevices] = {};
  if (dev < kMaxDevices && max_pairs[dev] == 0) {
    cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
    if (e != cudaSuccess) return set_cuda_error("cudaFuncSetAttribute(w8 kernel)", e);
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
  W8Maps maps;
  W8Group grp;
  memset(&maps, 0, sizeof(maps));
  memset(&grp, 0, sizeof(grp));
  grp.nprob = nprob;
  int max_tiles = 0;
  for (int j = 0; j < nprob; ++j) {
    const W8Problem& pr = prs[j];
    int rc = encode_tmap_2d(&maps.x[j], dt, 2, pr.x, pr.K, pr.M, pr.x_row_stride, C::BK, C::BM,
                            CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    rc = encode_tmap_2d(&maps.q[j], CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, pr.wq, pr.K, pr.N,
                        pr.wq_row_stride, C::BK, C::BN_HALF, CU_TENSOR_MAP_SWIZZLE_64B);
    if (rc) return rc;
    rc = encode_tmap_2d(&maps.out[j], dt, 2, pr.out, pr.N, pr.M, pr.out_row_stride, 64, 32,
                        CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    if (C::HALF_TAIL) {
      rc = encode_tmap_2d(&maps.out_half[j], dt, 2, pr.out, pr.N, pr.M, pr.out_row_stride, 32, 32,
                          CU_TENSOR_MAP_SWIZZLE_64B);
      if (rc) return rc;
    } else {
      maps.out_half[j] = maps.out[j];
    }
    W8Params& p = grp.p[j];
    p.M = static_cast<int32_t>(pr.M);
    p.N = static_cast<int32_t>(pr.N);
    p.K = static_cast<int32_t>(pr.K);
    p.num_m_blocks = static_cast<int32_t>((pr.M + 2 * C::BM - 1) / (2 * C::BM));
    p.num_n_blocks = static_cast<int32_t>((pr.N + BN - 1) / BN);
    p.num_k_blocks = static_cast<int32_t>((pr.K + C::BK - 1) / C::BK);
    p.eps = pr.eps;
    p.scale = pr.scale;
    p.bias = pr.bias;
    p.out = pr.out;
    p.out_row_stride = pr.out_row_stride;
    p.timeout_ns = wait_timeout_ns();
    const int tiles = p.num_m_blocks * p.num_n_blocks;
    if (tiles > max_tiles) max_tiles = tiles;
  }
  // As many pairs as the larger problem has tiles (the smaller one's runs
  // then sit on the last pairs, away from the larger one's extra tiles).
  const int pairs = max_tiles < pairs_avail ? max_tiles : pairs_avail;
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
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, maps, grp);
  if (e != cudaSuccess) return set_cuda_error("launch fused_rmsnorm_linear_w8", e);
  return 0;
}

// Tile width for the int8 kernel: the fewest tensor-core MACs on the busiest
// pair, sum over the problems of ceil(tiles / pairs) * bn * k-blocks (ties to
// the wider tile); 256 leaves room for only six int8 slots instead of eight.
static int choose_w8_bn(const W8Problem* prs, int nprob, int pairs) {
  static const int cands[] = {256, 224, 192, 128};
  int pick = 256;
  double best = 1e300;
  for (int bn : cands) {
    double cost = 0.0;
    for (int j = 0; j < nprob; ++j) {
      const int64_t mb = (prs[j].M + 255) / 256;
      const int64_t tiles = mb * ((prs[j].N + bn - 1) / bn);
      const int64_t nkb = (prs[j].K + 63) / 64;
      cost += static_cast<double>((tiles + pairs - 1) / pairs) * bn * static_cast<double>(nkb);
    }
    cost *= (bn == 256 ? 1.1 : 1.0);  // the shallower ring
    if (cost < best * 0.999) { best = cost; pick = bn; }
  }
  return pick;
}

template <typename T>
static int run_w8_t(const W8Problem* prs, int nprob, cudaStream_t s) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return set_cuda_error("cudaGetDevice");
  switch (choose_w8_bn(prs, nprob, sm_count(dev) / 2)) {
    case 256: return launch_w8<T, 256, 4, 6>(prs, nprob, s);
    case 224: return launch_w8<T, 224, 5, 5>(prs, nprob, s);
    case 192: return launch_w8<T, 192, 5, 6>(prs, nprob, s);
    default: return launch_w8<T, 128, 6, 8>(prs, nprob, s);
  }
}

int run_fused_linear_w8_group(const W8Problem* prs, int nprob, cudaStream_t s) {
  if (nprob < 1 || nprob > 2)
    return set_error(FRN_ERR_INVALID_ARGUMENT, "one launch takes 1 or 2 problems (got %d)", nprob);
  for (int j = 1; j < nprob; ++j)
    if (prs[j].dtype != prs[0].dtype)
      return set_error(FRN_ERR_INVALID_ARGUMENT, "grouped problems must share one dtype");
  if (prs[0].dtype != FRN_DTYPE_BF16 && prs[0].dtype != FRN_DTYPE_F16)
    return set_error(FRN_ERR_UNSUPPORTED, "int8-weight RMSNorm+Linear takes bf16 or fp16 x");
  // One launch pays off while each problem is one 256-row m-block (per-launch
  // start and last epilogue dominate: 33.2 -> 25.4 us for Kimi q_b + kv_b at
  // 256 rows); with more rows the shared tile width costs what the saved
  // launch gains, so each problem gets its own launch and tile width.
  if (nprob == 2 && (prs[0].M > 256 || prs[1].M > 256)) {
    const int rc = run_fused_linear_w8_group(&prs[0], 1, s);
    return rc ? rc : run_fused_linear_w8_group(&prs[1], 1, s);
  }
  if (prs[0].dtype == FRN_DTYPE_BF16) return run_w8_t<__nv_bfloat16>(prs, nprob, s);
  return run_w8_t<__half>(prs, nprob, s);
}

int run_fused_linear_w8(const W8Problem& pr, cudaStream_t s) {
  return run_fused_linear_w8_group(&pr, 1, s);
}

}  // namespace frn
