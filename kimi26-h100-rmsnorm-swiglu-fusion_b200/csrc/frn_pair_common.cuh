// frn_pair_common.cuh -- pieces shared by the SM-pair (cta_group::2) kernels:
// launch parameters, output tensor maps, and the TMA-store epilogue of one
// linear tile.
#pragma once

#include <cuda.h>

#include <cstdint>

#include "frn_internal.h"
#include "frn_ptx.cuh"

namespace frn {

// Output tensor maps: [32 rows x 64 columns] store boxes (128B swizzle), one
// per output part, plus a [32 x 32] box (64B swizzle) for tiles whose last
// chunk is 32 columns wide (single output only).
struct PairOut {
  CUtensorMap map[kMaxParts];
  CUtensorMap half;
  int32_t col0[kMaxParts];  // first output column of each part
  int32_t nparts;
};

struct PairParams {
  int32_t M, N, K;
  int32_t num_m_blocks;  // of 256 rows
  int32_t num_n_blocks;  // of BN columns
  int32_t num_k_blocks;  // of 64
  float eps;
  const void* bias;  // may be null
  void* out;
  int64_t out_row_stride;  // elements
  int32_t up_row0;         // SwiGLU: first W row of the up block (= intermediate)
  uint64_t timeout_ns;
};

// Output tensor maps of a pair kernel launch: one [32 x 64] 128B-swizzled
// store box per output part (the plain output is one part), and, for tiles
// whose last chunk is 32 columns wide (`half_tail`), a [32 x 32] 64B-swizzled
// box of the plain output.
inline int build_pair_out(const LinearProblem& pr, int64_t n_out, bool half_tail,
                          PairOut* outm) {
  const CUtensorMapDataType dt = pr.dtype == FRN_DTYPE_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                           : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  int rc = 0;
  if (pr.parts && pr.parts->n > 1) {
    if (half_tail)
      return set_error(FRN_ERR_UNSUPPORTED, "split output needs a tile width multiple of 64");
    outm->nparts = pr.parts->n;
    for (int i = 0; i < pr.parts->n; ++i) {
      rc = encode_tmap_2d(&outm->map[i], dt, 2, pr.parts->out[i], pr.parts->cols[i], pr.M,
                          pr.parts->stride[i], 64, 32, CU_TENSOR_MAP_SWIZZLE_128B);
      if (rc) return rc;
      outm->col0[i] = static_cast<int32_t>(pr.parts->col0[i]);
    }
    outm->half = outm->map[0];
  } else {
    outm->nparts = 1;
    outm->col0[0] = 0;
    rc = encode_tmap_2d(&outm->map[0], dt, 2, pr.out, n_out, pr.M, pr.out_row_stride, 64, 32,
                        CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    if (half_tail) {
      rc = encode_tmap_2d(&outm->half, dt, 2, pr.out, n_out, pr.M, pr.out_row_stride, 32, 32,
                          CU_TENSOR_MAP_SWIZZLE_64B);
      if (rc) return rc;
    } else {
      outm->half = outm->map[0];
    }
  }
  for (int i = outm->nparts; i < kMaxParts; ++i) {
    outm->map[i] = outm->map[0];
    outm->col0[i] = 0x7fffffff;
  }
  return 0;
}

// Epilogue of one linear pair tile, `width` (<= TILE_N, a multiple of 32)
// columns wide, for a warp whose TMEM lane quarter holds rows row_base ..
// row_base+31 of this CTA's half (taddr points at that quarter of the
// accumulator): for each 64-column chunk c (the last may be 32 wide) with c % chunk_mod == chunk_sel, TMEM -> fp32 -> acc * inv_rms (+ b)
// -> one rounding -> 128B-swizzled [32 x 64] smem block (double-buffered at
// stg + (nst % 2) * 4 KB) -> TMA tensor store through the output part's map,
// which also clips rows >= M and columns >= N.  After its last TMEM read the
// warp releases the accumulator on `tmem_empty_remote` (the even CTA's
// barrier) if `release_acc`.
template <typename T, int TILE_N>
__device__ __forceinline__ void pair_store_linear_tile(uint8_t* stg, uint32_t lane,
                                                       uint32_t taddr, int n0, int row_base,
                                                       float inv_rms, const T* bias, int N,
                                                       const PairOut& outm, uint32_t& nst,
                                                       bool release_acc,
                                                       uint32_t tmem_empty_remote,
                                                       int chunk_mod = 1, int chunk_sel = 0,
                                                       int width = TILE_N) {
  const int nchunk = (width + 63) / 64;
  const bool half_tail = width % 64 != 0;
  constexpr int STG_BYTES = 32 * 128;
  const bool has_bias = bias != nullptr;
  int c_last = nchunk - 1;  // this warp's last chunk
  while (c_last % chunk_mod != chunk_sel) --c_last;
#pragma unroll 1
  for (int c = chunk_sel; c < nchunk; c += chunk_mod, ++nst) {
    const bool half = half_tail && c == nchunk - 1;
    const int col0 = n0 + c * 64;
    uint4 bv[8];
    if (has_bias) {
#pragma unroll
      for (int j = 0; j < 8; ++j)
        bv[j] = (col0 + j * 8 < N && !(half && j >= 4)) ? ld_global_nc_v4(bias + col0 + j * 8)
                                                         : make_uint4(0u, 0u, 0u, 0u);
    }
    uint32_t v[64];
    tmem_ld_32x32b_x32(taddr + c * 64, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
    if (!half) tmem_ld_32x32b_x32(taddr + c * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
    tmem_ld_wait();
    if (c == c_last && release_acc) {
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster_relaxed(tmem_empty_remote);
    }
    uint8_t* sbp = stg + (nst & 1u) * STG_BYTES;
    const uint32_t sb = smem_addr(sbp);
    // The TMA store issued two chunks ago read this buffer; at most the
    // previous chunk's store may still be reading smem.
    if (lane == 0) bulk_wait_group_read<1>();
    __syncwarp();
    if (half) {
      if (has_bias) stage_rows_swizzled<T, 4, true>(v, inv_rms, bv, sb, lane);
      else stage_rows_swizzled<T, 4, false>(v, inv_rms, bv, sb, lane);
    } else {
      if (has_bias) stage_rows_swizzled<T, 8, true>(v, inv_rms, bv, sb, lane);
      else stage_rows_swizzled<T, 8, false>(v, inv_rms, bv, sb, lane);
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      // A chunk never straddles two parts: split outputs take 64-column
      // multiples for parts and tiles.
      int pi = 0;
      while (pi + 1 < outm.nparts && col0 >= outm.col0[pi + 1]) ++pi;
      tma_store_2d(half ? &outm.half : &outm.map[pi], sbp, col0 - outm.col0[pi], row_base);
      bulk_commit_group();
    }
  }
}

}  // namespace frn
