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
//   reduce    token t belongs to CTA t % S.  Once its MMAs are done, each
//             CTA pushes its fp32 partial D^T column of every token, and its
//             partial sum of x^2, into the owner's receive buffer
//             (st.shared::cluster; remote stores do not wait, remote loads
//             would); after one release/acquire cluster barrier each owner
//             sums its tokens' S partials from local shared memory in rank
//             order (deterministic, no atomics, no global workspace), applies
//             inv_rms[t] = rsqrt(sum_s ss_s[t] / K + eps) and b[n], and
//             stores out[t, n0 .. n0+127] as coalesced rows.
//
// SwiGLU variant: a tile is 64 gate rows over the matching 64 up rows, and
// the reduction combines the two halves into 64 output columns.
//
// Roles: warps 0-3 epilogue, warps 4-7 TMA producers (W / x over even / odd
// stages), warps 8 and 13 MMA issuers of the even / odd k-blocks into two
// accumulators (warp 8 also owns TMEM), warps 9-12 RMS (x^2 sums from the x
// stages, 16-byte chunks spread over all 128 threads).  Warps 0-7 then move
// the accumulators out of TMEM and push them, and reduce the owned tokens.
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
  static constexpr int PIPE_BYTES = STAGES * (W_BYTES + X_BYTES);
  // Receive buffer of the cluster reduction: fp32 [source rank][owned token
  // slot][W row].  An owner holds ceil(MP / S) token slots per source rank,
  // S * ceil(MP / S) <= MP + 7 for S <= 8.  Its own space when that fits
  // beside the pipeline, else it reuses the W stages (after every CTA of the
  // cluster has finished its MMAs).
  static constexpr int RECV_BYTES = (MP + 8) * BM * 4;
  static constexpr int SS_BYTES = (MP + 8) * 4;  // [source rank][owned token slot] sums of x^2
  static constexpr int NUM_BARS = 2 * STAGES + 3;
  static constexpr int TAIL_BYTES = SS_BYTES + NUM_BARS * 8 + 16 + 1024;
  static constexpr bool RECV_OWN = PIPE_BYTES + RECV_BYTES + TAIL_BYTES <= 232448;
  static constexpr int OFF_RECV = RECV_OWN ? PIPE_BYTES : 0;
  static constexpr int OFF_SS = RECV_OWN ? PIPE_BYTES + RECV_BYTES : PIPE_BYTES;
  static constexpr int OFF_BAR = OFF_SS + SS_BYTES;
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
  static constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;
  // warps 4-7: producers (W | x) x (even | odd stages); 8, 13: MMA; 9-12: RMS
  static constexpr int WARP_PROD0 = 4, WARP_MMA = 8, WARP_RMS0 = 9, WARP_MMA1 = 13;
  static constexpr int THREADS = 32 * 14;
  static_assert(STAGES % 2 == 0, "stages alternate between two producers and two issuers");
  static_assert(MP % 16 == 0 && MP >= 16 && MP <= 128, "MP");
  static_assert(X_BYTES % 1024 == 0, "x stages must stay 1024-aligned");
  static_assert(RECV_OWN || RECV_BYTES <= STAGES * W_BYTES,
                "a shared receive buffer may only overlap the W stages");
  static_assert(OFF_BAR % 8 == 0, "mbarriers need 8-byte alignment");
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
  float* recv = reinterpret_cast<float*>(smem + C::OFF_RECV);
  float* ss_recv = reinterpret_cast<float*>(smem + C::OFF_SS);

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
  // Cluster rendezvous A guards the first write into a peer's shared memory.
  // With a receive buffer of its own, a CTA is ready for its peers' writes
  // once it has started, so A is taken now (a warp that took it only after
  // its mainloop work waited ~0.4 us there); otherwise every CTA arrives once
  // its pipeline buffers are no longer read (below).
  if (C::RECV_OWN) {
    cluster_arrive_relaxed();
    cluster_wait();
  }
  bool acc_ready = false;
  float rms_ss[MP / 16];  // RMS warps: per-token partial sums of x^2 of this lane's chunk
#pragma unroll
  for (int i = 0; i < MP / 16; ++i) rms_ss[i] = 0.f;
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
      // Warm L2 with this thread's first two rings of tiles while the
      // preceding grid drains (see tma_prefetch_2d); two rings measured
      // 0.1-0.4 us faster than one over M = 1..128, more TMA prefetches
      // slower (they share the SM's TMA issue slots with the loads).
      for (int i = static_cast<int>(parity_sel); i < nkb && i < 2 * STAGES; i += 2) {
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
    // The producer warps help the epilogue warps move the accumulators out.
    __syncwarp();
    acc_ready = mbar_wait(tmem_full, 0, abort_flag, to);
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
    // The x stage's MP rows x 8 16-byte chunks are spread over the 128
    // threads: thread tid takes chunk tid % 8 of tokens i * 16 + tid / 8, so
    // every thread has work at any MP (one warp doing all of a small batch
    // fell ~1 us behind the stream).  The 8 chunk sums of a token are
    // combined with shuffles after the loop.
    const int tid = static_cast<int>(threadIdx.x) - C::WARP_RMS0 * 32;
    const uint32_t q = static_cast<uint32_t>(tid) & 7u;
    const int g = tid >> 3;
    uint32_t stage = 0, phase = 0;
    for (int i = 0; i < nkb; ++i) {
      if (!mbar_wait(&full[stage], phase, abort_flag, to)) break;
      const uint32_t xs = smem_addr(smem + C::OFF_X + stage * C::X_BYTES);
#pragma unroll
      for (int j = 0; j < MP / 16; ++j) {
        const uint32_t t = static_cast<uint32_t>(j * 16 + g);
        const uint4 v = ld_shared_v4(xs + t * 128u + ((q ^ (t & 7u)) << 4));
        const float2 f0 = pair_to_float2<T>(v.x), f1 = pair_to_float2<T>(v.y);
        const float2 f2 = pair_to_float2<T>(v.z), f3 = pair_to_float2<T>(v.w);
        float a = rms_ss[j];
        a = fmaf(f0.x, f0.x, a); a = fmaf(f0.y, f0.y, a);
        a = fmaf(f1.x, f1.x, a); a = fmaf(f1.y, f1.y, a);
        a = fmaf(f2.x, f2.x, a); a = fmaf(f2.y, f2.y, a);
        a = fmaf(f3.x, f3.x, a); a = fmaf(f3.y, f3.y, a);
        rms_ss[j] = a;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[stage]);
      if (++stage == STAGES) { stage = 0; phase ^= 1u; }
    }
#pragma unroll
    for (int j = 0; j < MP / 16; ++j) {
      float a = rms_ss[j];
      a += __shfl_xor_sync(0xffffffffu, a, 1);
      a += __shfl_xor_sync(0xffffffffu, a, 2);
      a += __shfl_xor_sync(0xffffffffu, a, 4);
      rms_ss[j] = a;
    }
  } else {
    // Epilogue warps 0-3: wait until every MMA of this CTA is done.
    acc_ready = mbar_wait(tmem_full, 0, abort_flag, to);
  }

  // Rendezvous A (shared receive buffer): every CTA of the cluster is done
  // with its W stages and can take its peers' writes.
  __syncwarp();
  tc_fence_before();
  if (!C::RECV_OWN) {
    cluster_arrive_release();  // after this CTA's last use of its W stages
    cluster_wait();
  }

  // Token t belongs to CTA t % S (slot t / S).  Each CTA writes its partial
  // D^T row of every token, and the RMS warps its partial sum of x^2, into
  // the owner's receive buffer at [this rank][slot], so that the reduction
  // below reads only local shared memory (remote loads cost a long round
  // trip each; remote stores do not wait).
  const int t_end = p.M < MP ? p.M : MP;
  const int towns = (MP + S - 1) / S;  // token slots per source rank
  if (warp < 8) {
    // Warps w and w + 4 share TMEM lane quarter w % 4 (W rows 32 (w % 4) ..)
    // and take alternate 16-token chunks.
    if (acc_ready) {
      tc_fence_after();
      const uint32_t quarter = warp & 3u;
      const uint32_t taddr = tmem_base + ((quarter * 32u) << 16);
      const uint32_t wrow = quarter * 32u + lane;
      const bool two = nkb >= 2;  // the odd issuer had k-blocks to accumulate
      const uint32_t mine =
          smem_addr(recv) + ((rank * static_cast<uint32_t>(towns)) * C::BM + wrow) * 4u;
#pragma unroll 1
      for (int c = static_cast<int>(warp >> 2); c < MP / 16 && c * 16 < t_end; c += 2) {
        int o = (c * 16) % S, tl = (c * 16) / S;  // owner and slot of token c * 16 + e
        uint32_t v[16], v1[16];
        tmem_ld_32x32b_x16(taddr + c * 16, v);
        if (two) tmem_ld_32x32b_x16(taddr + MP + c * 16, v1);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          if (c * 16 + e < t_end) {
            const uint32_t a = mine + static_cast<uint32_t>(tl) * (C::BM * 4u);
            const float val = __uint_as_float(v[e]) + (two ? __uint_as_float(v1[e]) : 0.f);
            st_shared_cluster_f32(mapa_shared(a, static_cast<uint32_t>(o)), val);
          }
          if (++o == S) { o = 0; ++tl; }
        }
      }
    }
  } else if (warp >= C::WARP_RMS0 && warp < C::WARP_RMS0 + 4) {
    const int tid = static_cast<int>(threadIdx.x) - C::WARP_RMS0 * 32;
    if ((tid & 7) == 0) {
#pragma unroll
      for (int j = 0; j < MP / 16; ++j) {
        const int t = j * 16 + (tid >> 3);
        if (t < t_end)
          st_shared_cluster_f32(
              mapa_shared(smem_addr(ss_recv) + static_cast<uint32_t>(rank * towns + t / S) * 4u,
                          static_cast<uint32_t>(t % S)),
              rms_ss[j]);
      }
    }
  }

  // Rendezvous B: every write into this CTA's receive buffer has landed.
  // Only warps 0-7 read TMEM since rendezvous A; the others' tcgen05 work was
  // fenced before it.
  __syncwarp();
  if (warp < 8) tc_fence_before();
  cluster_sync_all();

  if (warp < 8 && !*abort_flag) {
    // CTA `rank` reduces its owned tokens t = rank + S * tl, tl < n_own, with
    // warps 0-7 (the epilogue and producer warps, idle by now).  First
    // inv_rms[t] = rsqrt(sum_s ss_s[t] / K + eps), once per token, into slot
    // [0][tl] of the x^2 receive buffer (a thread reads only its own token's
    // slots); then TPT threads per token, each owning 4 output columns of the
    // tile (W rows pc .. pc+3, and for SwiGLU also the up rows 64+pc ..).
    constexpr int RT = 256;                   // reducing threads
    constexpr int OUTC = SWIGLU ? 64 : 128;   // output columns per tile
    constexpr int TPT = OUTC / 4;             // threads per token
    constexpr int LANES = RT / TPT;           // tokens in flight
    constexpr int kBatch = 2;
    const int tid = static_cast<int>(threadIdx.x);
    const int n_own = t_end > static_cast<int>(rank) ? (t_end - static_cast<int>(rank) + S - 1) / S : 0;
    const uint32_t recv_a = smem_addr(recv), ss_a = smem_addr(ss_recv);
    // Kernel parameters the loops need, in registers.
    const float kf = static_cast<float>(p.K), eps = p.eps;
    for (int tl = tid; tl < n_own; tl += RT) {
      float ss = 0.f;
      for (int s = 0; s < S; ++s)  // fixed rank order: deterministic sums
        ss += ld_shared_f32(ss_a + static_cast<uint32_t>(s * towns + tl) * 4u);
      ss_recv[tl] = rsqrtf(ss / kf + eps);
    }
    named_bar_sync(1, RT);
    griddep_wait();
    const int pc = (tid % TPT) * 4;
    const int tsub = tid / TPT;
    const bool col_ok = n0 + pc < p.N;  // N and part widths are multiples of 8
    int pi = 0;  // output part of columns n0 + pc .. n0 + pc + 3
    while (pi + 1 < p.nparts && n0 + pc >= p.part_col0[pi + 1]) ++pi;
    T* const obase = static_cast<T*>(p.part_out[pi]) + (n0 + pc - p.part_col0[pi]);
    const int64_t ostride = p.part_stride[pi];
    float bg[4] = {0.f, 0.f, 0.f, 0.f}, bu[4] = {0.f, 0.f, 0.f, 0.f};
    if (p.bias != nullptr && col_ok) {
      const T* bias = static_cast<const T*>(p.bias);
      const uint2 b = *reinterpret_cast<const uint2*>(bias + n0 + pc);
      const float2 b01 = pair_to_float2<T>(b.x), b23 = pair_to_float2<T>(b.y);
      bg[0] = b01.x; bg[1] = b01.y; bg[2] = b23.x; bg[3] = b23.y;
      if (SWIGLU) {
        const uint2 c = *reinterpret_cast<const uint2*>(bias + p.up_row0 + n0 + pc);
        const float2 c01 = pair_to_float2<T>(c.x), c23 = pair_to_float2<T>(c.y);
        bu[0] = c01.x; bu[1] = c01.y; bu[2] = c23.x; bu[3] = c23.y;
      }
    }
    for (int tl0 = tsub; tl0 < n_own; tl0 += LANES * kBatch) {
      float4 acc[kBatch], accu[kBatch];
      float r[kBatch];
#pragma unroll
      for (int j = 0; j < kBatch; ++j) {
        acc[j] = make_float4(0.f, 0.f, 0.f, 0.f);
        accu[j] = make_float4(0.f, 0.f, 0.f, 0.f);
        const int tl = tl0 + j * LANES;
        r[j] = ld_shared_f32(ss_a + static_cast<uint32_t>(tl < n_own ? tl : tl0) * 4u);
      }
      for (int s = 0; s < S; ++s) {  // fixed rank order: deterministic sums
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
          const int tl = tl0 + j * LANES;
          const int tc = tl < n_own ? tl : tl0;  // clamp: loads stay on written slots
          const uint32_t slot = recv_a + static_cast<uint32_t>((s * towns + tc) * C::BM + pc) * 4u;
          const float4 v = ld_shared_v4f(slot);
          acc[j].x += v.x; acc[j].y += v.y; acc[j].z += v.z; acc[j].w += v.w;
          if (SWIGLU) {
            const float4 u = ld_shared_v4f(slot + 64 * 4);
            accu[j].x += u.x; accu[j].y += u.y; accu[j].z += u.z; accu[j].w += u.w;
          }
        }
      }
#pragma unroll
      for (int j = 0; j < kBatch; ++j) {
        const int tl = tl0 + j * LANES;
        if (tl < n_own && col_ok) {
          const int t = static_cast<int>(rank) + S * tl;
          float y[4] = {acc[j].x * r[j] + bg[0], acc[j].y * r[j] + bg[1],
                        acc[j].z * r[j] + bg[2], acc[j].w * r[j] + bg[3]};
          if (SWIGLU) {
            const float u[4] = {accu[j].x, accu[j].y, accu[j].z, accu[j].w};
#pragma unroll
            for (int e = 0; e < 4; ++e)
              y[e] = __fdividef(y[e], 1.0f + __expf(-y[e])) * (u[e] * r[j] + bu[e]);
          }
          *reinterpret_cast<uint2*>(obase + static_cast<int64_t>(t) * ostride) =
              make_uint2(float2_to_pair<T>(y[0], y[1]), float2_to_pair<T>(y[2], y[3]));
        }
      }
    }
  }

  // No CTA touches a peer's shared memory after rendezvous B, so CTAs leave
  // without another cluster barrier.
  __syncwarp();
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
