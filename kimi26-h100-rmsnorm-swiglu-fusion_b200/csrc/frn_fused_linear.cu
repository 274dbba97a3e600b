// frn_fused_linear.cu -- fused RMSNorm -> Linear for sm_100a, prefill shapes.
//
// out[M,N] = round(inv_rms[m] * (x[M,K] . W[N,K]^T) + b[N]),
// inv_rms[m] = rsqrt(sum_k x[m,k]^2 / K + eps).
//
// This replaces the reference's two launches -- cuBLAS F.linear producing a
// rounded bf16 [M,N] and the in-place rmsnorm_normalize(_512) kernel that
// re-reads and rewrites it (reference src/fused_forward.py:182-191,
// csrc/denominator_kernel.cu:1202-1273) -- with ONE persistent kernel:
//
//   warp 4      TMA producer: x tile [128 x 64] and W tile [BN x 64] per
//               k-block into a STAGES-deep 128B-swizzled smem ring.
//   warp 5      TMEM owner + single-thread tcgen05.mma issuer (M=128, N=BN,
//               K=16 per instruction), fp32 accumulator double-buffered in
//               TMEM so tile i+1's mainloop overlaps tile i's epilogue.
//   warps 6-9   RMS reducers: thread t sums x[m0+t, :]^2 straight from the
//               same smem stages the MMA consumes, so x leaves HBM once and
//               the reduction costs no extra global traffic.  They release
//               each stage together with the MMA (empty barrier count 1+4).
//   warps 0-3   epilogue: tcgen05.ld of the accumulator (warp q owns TMEM
//               lanes 32q..32q+31 = tile rows), acc * inv_rms + b in fp32,
//               one rounding, 128B-swizzled smem staging, TMA store.
//
// Tiles are 128 x BN (BN in {128, 192, 256}), visited m-fastest so the CTAs
// that share a W tile run together and read it from HBM once.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>

#include "frn_internal.h"
#include "frn_ptx.cuh"

namespace frn {

struct FusedLinearParams {
  int32_t M, N, K;
  int32_t num_m_blocks, num_n_blocks, num_k_blocks;
  float eps;
  const void* bias;  // may be null
  uint64_t timeout_ns;
};

template <int BN, int STAGES>
struct FusedLinearCfg {
  static constexpr int BM = 128;
  static constexpr int BK = 64;  // 64 x 16-bit = one 128-byte swizzle row
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_TX = A_BYTES + B_BYTES;
  static constexpr int EPI_WARPS = 4;
  static constexpr int RMS_WARPS = 4;
  static constexpr int STG_BYTES = 32 * 128;  // 32 rows x 64 cols x 2 B
  static constexpr int STG_BUFS = 2;
  static constexpr uint32_t TMEM_COLS = (2 * BN <= 256) ? 256u : 512u;
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = OFF_A + STAGES * A_BYTES;
  static constexpr int OFF_STG = OFF_B + STAGES * B_BYTES;
  static constexpr int OFF_RMS = OFF_STG + EPI_WARPS * STG_BUFS * STG_BYTES;
  static constexpr int OFF_BAR = OFF_RMS + 2 * BM * 4;
  static constexpr int NUM_BARS = 2 * STAGES + 8 + 1;
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
  static constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;  // + base alignment slack
  static constexpr int THREADS = 32 * (EPI_WARPS + 2 + RMS_WARPS);
  static constexpr int WARP_PRODUCER = 4;
  static constexpr int WARP_MMA = 5;
  static constexpr int WARP_RMS0 = 6;
  static_assert(B_BYTES % 1024 == 0, "stage buffers must stay 1024-aligned");
  static_assert(BN % 64 == 0 && BN >= 64 && BN <= 256, "BN");
  static_assert(SMEM_BYTES <= 232448, "exceeds 227 KB of dynamic shared memory");
};

template <typename T, int BN, int STAGES>
__global__ void __launch_bounds__(FusedLinearCfg<BN, STAGES>::THREADS, 1)
    fused_rmsnorm_linear_kernel(const __grid_constant__ CUtensorMap tmap_x,
                                const __grid_constant__ CUtensorMap tmap_w,
                                const __grid_constant__ CUtensorMap tmap_out,
                                const FusedLinearParams p) {
  using C = FusedLinearCfg<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));

  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* empty = full + STAGES;
  uint64_t* tmem_full = empty + STAGES;
  uint64_t* tmem_empty = tmem_full + 2;
  uint64_t* rms_full = tmem_empty + 2;
  uint64_t* rms_empty = rms_full + 2;
  uint64_t* mma_done = rms_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile uint32_t* abort_flag = tmem_slot + 1;
  float* rms_buf = reinterpret_cast<float*>(smem + C::OFF_RMS);

  const uint32_t warp = warp_id_in_cta();
  const uint32_t lane = threadIdx.x & 31u;

  if (warp == C::WARP_PRODUCER && lane == 0) {
    prefetch_tmap(&tmap_x);
    prefetch_tmap(&tmap_w);
    prefetch_tmap(&tmap_out);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1 + C::RMS_WARPS);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tmem_full[a], 1);
      mbar_init(&tmem_empty[a], C::EPI_WARPS);
      mbar_init(&rms_full[a], C::RMS_WARPS);
      mbar_init(&rms_empty[a], C::EPI_WARPS);
    }
    mbar_init(mma_done, 1);
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

  const int num_tiles = p.num_m_blocks * p.num_n_blocks;
  const int nkb = p.num_k_blocks;
  const uint64_t to = p.timeout_ns;

  if (warp == C::WARP_PRODUCER) {
    if (lane == 0) {
      uint32_t stage = 0, phase = 0;
      uint32_t fills = 0;
      for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
        const int m0 = (t % p.num_m_blocks) * C::BM;
        const int n0 = (t / p.num_m_blocks) * BN;
        bool ok = true;
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, to)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[stage], C::STAGE_TX);
          tma_load_2d(smem + C::OFF_A + stage * C::A_BYTES, &tmap_x, &full[stage], kb * C::BK, m0);
          tma_load_2d(smem + C::OFF_B + stage * C::B_BYTES, &tmap_w, &full[stage], kb * C::BK, n0);
          ++fills;
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
      }
      // Never leave the CTA with TMA writes into its smem still in flight:
      // wait (bounded, ignoring the abort flag) for the last fill of each stage.
      uint32_t zero = 0;
      for (uint32_t s = 0; s < static_cast<uint32_t>(STAGES) && s < fills; ++s) {
        const uint32_t last = s + STAGES * ((fills - 1 - s) / STAGES);
        mbar_wait(&full[s], (last / STAGES) & 1u, &zero, to);
      }
    }
  } else if (warp == C::WARP_MMA) {
    if (lane == 0) {
      const uint32_t idesc = make_idesc_f16(Elem16<T>::kUmmaFormat, C::BM, BN);
      uint32_t stage = 0, phase = 0;
      int i = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++i) {
        const uint32_t acc = i & 1, acc_phase = (i >> 1) & 1;
        if (!mbar_wait(&tmem_empty[acc], acc_phase ^ 1u, abort_flag, to)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, to)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_addr(smem + C::OFF_A + stage * C::A_BYTES);
          const uint32_t b_addr = smem_addr(smem + C::OFF_B + stage * C::B_BYTES);
#pragma unroll
          for (int k = 0; k < C::BK / 16; ++k) {
            umma_f16_ss(d_tmem, make_smem_desc_k_sw128(a_addr + k * 32),
                        make_smem_desc_k_sw128(b_addr + k * 32), idesc,
                        (kb > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        umma_commit(&tmem_full[acc]);
      }
      // All issued MMAs must have retired before TMEM is released.
      umma_commit(mma_done);
      uint32_t zero = 0;
      mbar_wait(mma_done, 0, &zero, to);
    }
  } else if (warp >= C::WARP_RMS0) {
    const int r = static_cast<int>(threadIdx.x) - C::WARP_RMS0 * 32;  // tile row 0..127
    const float inv_k = 1.0f / static_cast<float>(p.K);
    uint32_t stage = 0, phase = 0;
    int i = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++i) {
      const uint32_t acc = i & 1, acc_phase = (i >> 1) & 1;
      float ss0 = 0.f, ss1 = 0.f;
      for (int kb = 0; kb < nkb; ++kb) {
        if (!mbar_wait(&full[stage], phase, abort_flag, to)) { ok = false; break; }
        const uint32_t row = smem_addr(smem + C::OFF_A + stage * C::A_BYTES) + r * 128;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          // logical 16-byte chunk q of this row sits at physical chunk q ^ (r % 8)
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
      if (!ok) break;
      if (!mbar_wait(&rms_empty[acc], acc_phase ^ 1u, abort_flag, to)) break;
      rms_buf[acc * C::BM + r] = rsqrtf((ss0 + ss1) * inv_k + p.eps);
      __syncwarp();
      if (lane == 0) mbar_arrive(&rms_full[acc]);
    }
  } else {
    // Epilogue warps 0..3: warp q reads TMEM lanes [32q, 32q+32) = tile rows.
    const uint32_t q = warp;
    const int row = static_cast<int>(q * 32 + lane);
    const bool has_bias = p.bias != nullptr;
    const uint4* bias16 = reinterpret_cast<const uint4*>(p.bias);
    uint32_t stg = 0;
    int i = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++i) {
      const uint32_t acc = i & 1, acc_phase = (i >> 1) & 1;
      const int m0 = (t % p.num_m_blocks) * C::BM;
      const int n0 = (t / p.num_m_blocks) * BN;
      if (!mbar_wait(&tmem_full[acc], acc_phase, abort_flag, to)) break;
      if (!mbar_wait(&rms_full[acc], acc_phase, abort_flag, to)) break;
      tc_fence_after();
      const float inv_rms = rms_buf[acc * C::BM + row];
      __syncwarp();
      if (lane == 0) mbar_arrive(&rms_empty[acc]);
      const uint32_t taddr = tmem_base + acc * BN + ((q * 32u) << 16);
#pragma unroll 1
      for (int c = 0; c < BN / 64; ++c) {
        uint32_t v0[32], v1[32];
        tmem_ld_32x32b_x32(taddr + c * 64, v0);
        tmem_ld_32x32b_x32(taddr + c * 64 + 32, v1);
        tmem_ld_wait();
        if (c == BN / 64 - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tmem_empty[acc]);
        }
        uint8_t* sb = smem + C::OFF_STG + (q * C::STG_BUFS + stg) * C::STG_BYTES;
        if (lane == 0) bulk_wait_group_read<C::STG_BUFS - 1>();
        __syncwarp();
        const int ncol0 = n0 + c * 64;
#pragma unroll
        for (int j = 0; j < 8; ++j) {  // 16-byte chunk j = columns [8j, 8j+8)
          float f[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const uint32_t bits = (j < 4) ? v0[j * 8 + e] : v1[(j - 4) * 8 + e];
            f[e] = __uint_as_float(bits) * inv_rms;
          }
          if (has_bias && ncol0 + j * 8 < p.N) {
            const uint4 bv = __ldg(bias16 + (ncol0 + j * 8) / 8);
            const float2 b0 = pair_to_float2<T>(bv.x), b1 = pair_to_float2<T>(bv.y);
            const float2 b2 = pair_to_float2<T>(bv.z), b3 = pair_to_float2<T>(bv.w);
            f[0] += b0.x; f[1] += b0.y; f[2] += b1.x; f[3] += b1.y;
            f[4] += b2.x; f[5] += b2.y; f[6] += b3.x; f[7] += b3.y;
          }
          uint4 o;
          o.x = float2_to_pair<T>(f[0], f[1]);
          o.y = float2_to_pair<T>(f[2], f[3]);
          o.z = float2_to_pair<T>(f[4], f[5]);
          o.w = float2_to_pair<T>(f[6], f[7]);
          *reinterpret_cast<uint4*>(sb + lane * 128 + ((j ^ (lane & 7)) << 4)) = o;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&tmap_out, sb, ncol0, m0 + static_cast<int>(q * 32));
          bulk_commit_group();
        }
        stg ^= 1u;
      }
    }
    if (lane == 0) bulk_wait_group_all();
  }

  __syncthreads();
  if (warp == C::WARP_MMA) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// ------------------------------------------------------------------ host side

template <typename T, int BN, int STAGES>
static int launch_fused_linear(const LinearProblem& pr, cudaStream_t stream) {
  using C = FusedLinearCfg<BN, STAGES>;
  auto kern = fused_rmsnorm_linear_kernel<T, BN, STAGES>;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return set_cuda_error("cudaGetDevice");
  static bool attr_set[kMaxDevices] = {};
  if (dev < kMaxDevices && !attr_set[dev]) {
    cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
    if (e != cudaSuccess) return set_cuda_error("cudaFuncSetAttribute(fused_rmsnorm_linear)", e);
    attr_set[dev] = true;
  }
  const CUtensorMapDataType dt = Elem16<T>::kTmaType;
  CUtensorMap tx, tw, to;
  int rc = encode_tmap_2d(&tx, dt, 2, pr.x, pr.K, pr.M, pr.x_row_stride, C::BK, C::BM,
                          CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = encode_tmap_2d(&tw, dt, 2, pr.w, pr.K, pr.N, pr.w_row_stride, C::BK, BN,
                      CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = encode_tmap_2d(&to, dt, 2, pr.out, pr.N, pr.M, pr.out_row_stride, 64, 32,
                      CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;

  FusedLinearParams p;
  p.M = static_cast<int32_t>(pr.M);
  p.N = static_cast<int32_t>(pr.N);
  p.K = static_cast<int32_t>(pr.K);
  p.num_m_blocks = static_cast<int32_t>((pr.M + C::BM - 1) / C::BM);
  p.num_n_blocks = static_cast<int32_t>((pr.N + BN - 1) / BN);
  p.num_k_blocks = static_cast<int32_t>((pr.K + C::BK - 1) / C::BK);
  p.eps = pr.eps;
  p.bias = pr.bias;
  p.timeout_ns = wait_timeout_ns();
  const int tiles = p.num_m_blocks * p.num_n_blocks;
  const int sms = sm_count(dev);
  const int grid = tiles < sms ? tiles : sms;
  kern<<<grid, C::THREADS, C::SMEM_BYTES, stream>>>(tx, tw, to, p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error("launch fused_rmsnorm_linear", e);
  return 0;
}

// Tile-width choice: minimise (tiles per CTA) x BN x (1 + 32/BN) -- the
// busiest CTA's MMA work, with a small charge for the extra operand traffic
// of narrower tiles -- over BN in {256, 192, 128}.
int choose_prefill_kernel(int64_t M, int64_t N, int sms) {
  const int64_t mb = (M + 127) / 128;
  const int bns[3] = {256, 192, 128};
  const int ids[3] = {3, 2, 1};
  double best = 1e300;
  int best_id = 3;
  for (int i = 0; i < 3; ++i) {
    const int64_t tiles = mb * ((N + bns[i] - 1) / bns[i]);
    const int64_t per_cta = (tiles + sms - 1) / sms;
    const double cost = static_cast<double>(per_cta) * (bns[i] + 32);
    if (cost < best - 1e-9) { best = cost; best_id = ids[i]; }
  }
  return best_id;
}

template <typename T>
static int run_prefill_t(const LinearProblem& pr, int kernel, cudaStream_t s) {
  switch (kernel) {
    case 1: return launch_fused_linear<T, 128, 6>(pr, s);
    case 2: return launch_fused_linear<T, 192, 4>(pr, s);
    case 3: return launch_fused_linear<T, 256, 4>(pr, s);
    default: return set_error(FRN_ERR_INVALID_ARGUMENT, "unknown prefill kernel id");
  }
}

int run_fused_linear_prefill(const LinearProblem& pr, int kernel, cudaStream_t s) {
  if (pr.dtype == FRN_DTYPE_BF16) return run_prefill_t<__nv_bfloat16>(pr, kernel, s);
  if (pr.dtype == FRN_DTYPE_F16) return run_prefill_t<__half>(pr, kernel, s);
  return set_error(FRN_ERR_UNSUPPORTED, "fused RMSNorm+Linear supports bf16 and fp16 only");
}

}  // namespace frn
