// frn_fused_linear_xres.cu -- SM-pair fused RMSNorm -> Linear with x resident
// in shared memory, for K <= 512 (Kimi kv_b: K = 512).
//
// The SM-pair kernel (frn_fused_linear_pair.cu) reloads the 128-row x tile of
// every k-block for every output tile, and the shared-memory port (TMA writes
// plus UMMA operand reads, 128 B/clk) is already the limit of a 256 x 224-256
// MMA.  When all of K fits (8 k-blocks x 16 KB = 128 KB per CTA), each CTA
// loads its 128 x K slice of x once per run of same-m-block tiles and keeps
// it; the ring then carries W half-tiles only, so per k-block the SM moves
// 16 KB (W) into and 32 KB (x, W) out of shared memory instead of 32 + 32,
// and inv_rms is reduced from the resident slice once per run.
//
// Roles (each CTA of the pair, 416 threads):
//   warps 0-3   epilogue (pair_store_linear_tile: TMEM -> bf16 -> TMA store)
//   warp 4      x loader: at each run start waits `a_empty`, then loads the
//               run's K/64 x k-blocks; both CTAs' loads complete on the even
//               CTA's `a_full[kb]`
//   warps 5, 6  W loaders (even / odd ring slots), completing on the even
//               CTA's `b_full[slot]`
//   warp 8      even CTA: MMA issuer; every CTA: TMEM owner.  In the first
//               tile of a run it forwards each `a_full[kb]` to both CTAs'
//               `a_ready[kb]` (a multicast commit), frees ring slots with a
//               multicast commit on `b_empty`, and after a run's last tile
//               commits `a_empty` in both CTAs
//   warps 9-12  RMS: per run, wait `a_ready[kb]` and sum x[row]^2 over the
//               resident slice, publish inv_rms, arrive `a_empty`
// Every multicast arrival is waited for by its target before the pair exits
// (the loaders drain the last `b_empty` / `a_empty` phases), so the exit
// rendezvous needs no release.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "frn_internal.h"
#include "frn_pair_common.cuh"
#include "frn_ptx.cuh"

namespace frn {

template <int BN, int BSTAGES>
struct XresCfg {
  static constexpr int BM = 128;
  static constexpr int BK = 64;
  static constexpr int MAX_KB = 8;  // K <= 512
  static constexpr int BN_HALF = BN / 2;
  static constexpr int A_BYTES = BM * BK * 2;       // one resident x k-block
  static constexpr int B_BYTES = BN_HALF * BK * 2;  // one W half-tile slot
  static constexpr int STG_BYTES = 32 * 128;
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = OFF_A + MAX_KB * A_BYTES;
  static constexpr int OFF_STG = OFF_B + BSTAGES * B_BYTES;
  static constexpr int OFF_RMS = OFF_STG + 4 * 2 * STG_BYTES;
  static constexpr int OFF_BAR = OFF_RMS + 2 * BM * 4;
  static constexpr int NUM_BARS = 2 * MAX_KB + 1 + 2 * BSTAGES + 9;
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
  static constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;
  static constexpr uint32_t TMEM_COLS = 2 * BN <= 256 ? 256u : 512u;
  static constexpr int WARP_ALOAD = 4, WARP_BLOAD0 = 5, WARP_MMA = 8, WARP_RMS0 = 9;
  static constexpr int THREADS = 32 * 13;
  static_assert(BSTAGES % 2 == 0, "slots are split between two W loaders");
  static_assert(B_BYTES % 1024 == 0 && OFF_STG % 1024 == 0, "1024-aligned buffers");
  static_assert(SMEM_BYTES <= 232448, "exceeds 227 KB of dynamic shared memory");
};

template <typename T, int BN, int BSTAGES>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(XresCfg<BN, BSTAGES>::THREADS, 1)
    fused_rmsnorm_linear_xres_kernel(const __grid_constant__ CUtensorMap tmap_x,
                                     const __grid_constant__ CUtensorMap tmap_w,
                                     const __grid_constant__ PairOut outm,
                                     const PairParams p) {
  using C = XresCfg<BN, BSTAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* a_full = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);  // even CTA
  uint64_t* a_ready = a_full + C::MAX_KB;
  uint64_t* a_empty = a_ready + C::MAX_KB;
  uint64_t* b_full = a_empty + 1;  // even CTA
  uint64_t* b_empty = b_full + BSTAGES;
  uint64_t* tmem_full = b_empty + BSTAGES;
  uint64_t* tmem_empty = tmem_full + 2;  // even CTA
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

  if (warp == C::WARP_ALOAD && lane == 0) {
    prefetch_tmap(&tmap_x);
    prefetch_tmap(&tmap_w);
    for (int i = 0; i < outm.nparts; ++i) prefetch_tmap(&outm.map[i]);
    for (int kb = 0; kb < C::MAX_KB; ++kb) {
      mbar_init(&a_full[kb], 1);
      mbar_init(&a_ready[kb], 1);
    }
    mbar_init(a_empty, 1 + 4);  // MMA commit + 4 RMS warps
    for (int s = 0; s < BSTAGES; ++s) {
      mbar_init(&b_full[s], 1);
      mbar_init(&b_empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tmem_full[a], 1);
      mbar_init(&tmem_empty[a], 8);
      mbar_init(&rms_full[a], 4);
      mbar_init(&rms_empty[a], 4);
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
  __syncthreads();
  cluster_sync_relaxed();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int num_tiles = p.num_m_blocks * p.num_n_blocks;
  const int tiles_base = num_tiles / static_cast<int>(num_pairs);
  const int tiles_rem = num_tiles % static_cast<int>(num_pairs);
  const int t_begin = static_cast<int>(pair) * tiles_base + min(static_cast<int>(pair), tiles_rem);
  const int t_end = t_begin + tiles_base + (static_cast<int>(pair) < tiles_rem ? 1 : 0);
  const int nkb = p.num_k_blocks;  // <= MAX_KB
  const int nnb = p.num_n_blocks;
  const uint64_t to = p.timeout_ns;
  griddep_launch_dependents();

  if (warp == C::WARP_ALOAD) {
    if (lane == 0) {
      griddep_wait();
      uint32_t runs = 0;
      int cur_m = -1;
      bool ok = true;
      for (int t = t_begin; t < t_end && ok; ++t) {
        const int mb = t / nnb;
        if (mb == cur_m) continue;
        cur_m = mb;
        if (!mbar_wait(a_empty, (runs & 1u) ^ 1u, abort_flag, to)) { ok = false; break; }
        const int m0 = mb * 2 * C::BM + static_cast<int>(rank) * C::BM;
        for (int kb = 0; kb < nkb; ++kb) {
          if (rank == 0) mbar_arrive_expect_tx(&a_full[kb], 2u * C::A_BYTES);
          tma_load_2d_pair(smem + C::OFF_A + kb * C::A_BYTES, &tmap_x,
                           mapa_shared(smem_addr(&a_full[kb]), 0), kb * C::BK, m0);
        }
        ++runs;
      }
      // The last run's release (a multicast commit) must land before exit.
      if (ok && runs > 0) mbar_wait(a_empty, (runs & 1u) ^ 1u, abort_flag, to);
    }
  } else if (warp == C::WARP_BLOAD0 || warp == C::WARP_BLOAD0 + 1) {
    if (lane == 0) {
      griddep_wait();
      const uint32_t sel = warp - C::WARP_BLOAD0;
      uint32_t stage = 0, phase = 0;
      bool ok = true;
      for (int t = t_begin; t < t_end && ok; ++t) {
        const int n0 = (t % nnb) * BN + static_cast<int>(rank) * C::BN_HALF;
        for (int kb = 0; kb < nkb; ++kb) {
          if ((stage & 1u) == sel) {
            if (!mbar_wait(&b_empty[stage], phase ^ 1u, abort_flag, to)) { ok = false; break; }
            if (rank == 0) mbar_arrive_expect_tx(&b_full[stage], 2u * C::B_BYTES);
            tma_load_2d_pair(smem + C::OFF_B + stage * C::B_BYTES, &tmap_w,
                             mapa_shared(smem_addr(&b_full[stage]), 0), kb * C::BK, n0);
          }
          if (++stage == BSTAGES) { stage = 0; phase ^= 1u; }
        }
      }
      // Drain: wait for the final release of each slot this thread fills, so
      // no multicast commit is still in flight when the pair exits.
      for (int j = 0; j < BSTAGES && ok; ++j) {
        if ((stage & 1u) == sel && !mbar_wait(&b_empty[stage], phase ^ 1u, abort_flag, to)) break;
        if (++stage == BSTAGES) { stage = 0; phase ^= 1u; }
      }
    }
  } else if (warp == C::WARP_MMA) {
    if (rank == 0 && lane == 0) {
      const uint32_t idesc = make_idesc_f16(Elem16<T>::kUmmaFormat, 2 * C::BM, BN);
      uint32_t stage = 0, phase = 0, run = 0;
      int cur_m = -1, i = 0;
      bool ok = true;
      for (int t = t_begin; t < t_end && ok; ++t, ++i) {
        const int mb = t / nnb;
        const bool first = mb != cur_m;
        if (first) {
          if (cur_m >= 0) ++run;
          cur_m = mb;
        }
        const bool last_of_run = (t + 1 >= t_end) || ((t + 1) / nnb != mb);
        const uint32_t acc = i & 1, acc_phase = (i >> 1) & 1;
        if (!mbar_wait_cluster(&tmem_empty[acc], acc_phase ^ 1u, abort_flag, to)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < nkb; ++kb) {
          if (first) {
            if (!mbar_wait(&a_full[kb], run & 1u, abort_flag, to)) { ok = false; break; }
            tc_fence_after();
            umma_commit_pair_mc(&a_ready[kb], 0x3);
          }
          if (!mbar_wait(&b_full[stage], phase, abort_flag, to)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_addr(smem + C::OFF_A + kb * C::A_BYTES);
          const uint32_t b_addr = smem_addr(smem + C::OFF_B + stage * C::B_BYTES);
#pragma unroll
          for (int k = 0; k < C::BK / 16; ++k)
            umma_f16_ss_pair(d_tmem, make_smem_desc_k_sw128(a_addr + k * 32),
                             make_smem_desc_k_sw128(b_addr + k * 32), idesc,
                             (kb > 0 || k > 0) ? 1u : 0u);
          umma_commit_pair_mc(&b_empty[stage], 0x3);
          if (++stage == BSTAGES) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        umma_commit_pair_mc(&tmem_full[acc], 0x3);
        if (last_of_run) umma_commit_pair_mc(a_empty, 0x3);
      }
      umma_commit_pair_mc(drain, 0x1);
      uint32_t zero = 0;
      mbar_wait(drain, 0, &zero, to);
    }
  } else if (warp >= C::WARP_RMS0) {
    const int r = static_cast<int>(threadIdx.x) - C::WARP_RMS0 * 32;
    const float inv_k = 1.0f / static_cast<float>(p.K);
    const uint32_t a0 = smem_addr(smem + C::OFF_A) + r * 128;
    uint32_t gen = 0;
    int cur_m = -1;
    for (int t = t_begin; t < t_end; ++t) {
      const int mb = t / nnb;
      if (mb == cur_m) continue;
      cur_m = mb;
      float ss0 = 0.f, ss1 = 0.f;
      bool ok = true;
      for (int kb = 0; kb < nkb; ++kb) {
        if (!mbar_wait(&a_ready[kb], gen & 1u, abort_flag, to)) { ok = false; break; }
        const uint32_t row = a0 + kb * C::A_BYTES;
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
      if (!ok) break;
      if (!mbar_wait(&rms_empty[gen & 1], ((gen >> 1) & 1u) ^ 1u, abort_flag, to)) break;
      rms_buf[(gen & 1) * C::BM + r] = rsqrtf((ss0 + ss1) * inv_k + p.eps);
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&rms_full[gen & 1]);
        mbar_arrive(a_empty);  // done reading this run's x slice
      }
      ++gen;
    }
  } else if (warp < 4) {
    const uint32_t q = warp;
    const T* bias = static_cast<const T*>(p.bias);
    const uint32_t leader_tmem_empty0 = mapa_shared(smem_addr(&tmem_empty[0]), 0);
    griddep_wait();
    uint32_t nst = 0;
    int i = 0, gen = -1, cur_m = -1;
    float inv_rms = 0.f;
    for (int t = t_begin; t < t_end; ++t, ++i) {
      const uint32_t acc = i & 1, acc_phase = (i >> 1) & 1;
      const int mb = t / nnb;
      const int row_base = mb * 2 * C::BM + static_cast<int>(rank) * C::BM + static_cast<int>(q) * 32;
      const int n0 = (t % nnb) * BN;
      const bool first = mb != cur_m;
      const bool last = (t + 1 >= t_end) || ((t + 1) / nnb != mb);
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
      pair_store_linear_tile<T, BN>(smem + C::OFF_STG + q * 2 * C::STG_BYTES, lane,
                                    tmem_base + acc * BN + ((q * 32u) << 16), n0, row_base,
                                    inv_rms, bias, p.N, outm, nst, t + 2 < t_end,
                                    leader_tmem_empty0 + acc * 8);
    }
    if (lane == 0) bulk_wait_group_read<0>();
  }

  __syncwarp();
  tc_fence_before();
  cluster_sync_relaxed();
  if (*abort_flag) __nanosleep(20000);
  if (warp == C::WARP_MMA) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
  }
}

// ------------------------------------------------------------------ host side

template <typename T, int BN, int BSTAGES>
static int launch_xres(const LinearProblem& pr, cudaStream_t stream) {
  using C = XresCfg<BN, BSTAGES>;
  auto kern = fused_rmsnorm_linear_xres_kernel<T, BN, BSTAGES>;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return set_cuda_error("cudaGetDevice");
  static int max_pairs[kMaxDevices] = {};
  if (dev < kMaxDevices && max_pairs[dev] == 0) {
    cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
    if (e != cudaSuccess) return set_cuda_error("cudaFuncSetAttribute(xres kernel)", e);
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
  PairOut outm;
  rc = build_pair_out(pr, pr.N, BN % 64 != 0, &outm);
  if (rc) return rc;
  PairParams p;
  p.M = static_cast<int32_t>(pr.M);
  p.N = static_cast<int32_t>(pr.N);
  p.K = static_cast<int32_t>(pr.K);
  p.num_m_blocks = static_cast<int32_t>((pr.M + 2 * C::BM - 1) / (2 * C::BM));
  p.num_n_blocks = static_cast<int32_t>((pr.N + BN - 1) / BN);
  p.num_k_blocks = static_cast<int32_t>((pr.K + C::BK - 1) / C::BK);
  p.eps = pr.eps;
  p.bias = pr.bias;
  p.out = pr.out;
  p.out_row_stride = pr.out_row_stride;
  p.up_row0 = 0;
  p.timeout_ns = wait_timeout_ns();
  if (p.num_k_blocks > C::MAX_KB)
    return set_error(FRN_ERR_UNSUPPORTED, "x-resident kernel takes K <= %d", C::MAX_KB * C::BK);
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
  if (e != cudaSuccess) return set_cuda_error("launch fused_rmsnorm_linear_xres", e);
  return 0;
}

// Tile width for the x-resident kernel: per pair tile nkb * 2 * BN cycles of
// MMA against nkb * BN * 64 B of W feed at ~60 B/clk per SM (x is loaded once
// per run), over ceil(tiles / pairs) tiles, plus the one exposed epilogue.
int choose_xres_bn(int64_t M, int64_t N, int64_t K, int pairs, bool tile64) {
  const double mb = static_cast<double>((M + 255) / 256);
  const double nkb = static_cast<double>((K + 63) / 64);
  static const int cands[] = {256, 224, 192, 128};
  double best = 1e300;
  int pick = 256;
  for (int bn : cands) {
    if (tile64 && bn % 64) continue;
    const double tiles = mb * std::ceil(static_cast<double>(N) / bn);
    const double per_pair = std::ceil(tiles / pairs);
    const double mma = nkb * 2.0 * bn;
    const double feed = nkb * bn * 64.0 / 60.0;
    const double epi = 128.0 * bn * 2.0 / 26.0;
    const double total = per_pair * (mma > feed ? mma : feed) + epi;
    if (total < best * 0.999) { best = total; pick = bn; }
  }
  return pick;
}

template <typename T>
static int run_xres_t(const LinearProblem& pr, int bn, cudaStream_t s) {
  switch (bn) {
    case 256: return launch_xres<T, 256, 4>(pr, s);
    case 224: return launch_xres<T, 224, 4>(pr, s);
    case 192: return launch_xres<T, 192, 4>(pr, s);
    case 128: return launch_xres<T, 128, 8>(pr, s);
    default: break;
  }
  return set_error(FRN_ERR_INVALID_ARGUMENT, "unsupported x-resident tile width %d", bn);
}

int run_fused_linear_xres(const LinearProblem& pr, int bn, cudaStream_t s) {
  if (pr.dtype == FRN_DTYPE_BF16) return run_xres_t<__nv_bfloat16>(pr, bn, s);
  if (pr.dtype == FRN_DTYPE_F16) return run_xres_t<__half>(pr, bn, s);
  return set_error(FRN_ERR_UNSUPPORTED, "fused RMSNorm+Linear supports bf16 and fp16 only");
}

}  // namespace frn
