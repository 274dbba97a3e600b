// frn_internal.h -- host-side helpers shared by the kernel launchers and the
// C ABI (frn_capi.cu).  Not part of the public interface.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "../../include/frn_b200.h"

namespace frn {

constexpr int kMaxDevices = 64;

// One fused RMSNorm -> Linear problem, validated by the C ABI before any
// launcher sees it.  Strides are in elements.
// Output columns [0, N) split into up to kMaxParts separate tensors: part p
// holds columns [col0[p], col0[p] + cols[p]) at out[p] with row stride
// stride[p] (elements).  One part = the plain [M, N] output.
constexpr int kMaxParts = 4;
struct OutParts {
  int n;
  int64_t col0[kMaxParts];
  int64_t cols[kMaxParts];
  void* out[kMaxParts];
  int64_t stride[kMaxParts];
};

struct LinearProblem {
  int dtype;
  const void* x;
  int64_t M, K, x_row_stride;
  const void* w;
  int64_t N, w_row_stride;
  const void* bias;  // may be null
  float eps;
  void* out;
  int64_t out_row_stride;
  void* workspace;
  size_t workspace_bytes;
  const OutParts* parts = nullptr;  // non-null: write the split parts instead of out
};

// One int8-weight problem (strides in elements; wq_row_stride in bytes).
struct W8Problem {
  int dtype;
  const void* x;
  int64_t M, K, x_row_stride;
  const int8_t* wq;
  int64_t N, wq_row_stride;
  const float* scale;
  const void* bias;
  float eps;
  void* out;
  int64_t out_row_stride;
};

// Records `msg` as this thread's last error and returns `code`.
int set_error(int code, const char* fmt, ...);
// Records a CUDA failure ("<what>: <cuda error string>") and returns FRN_ERR_CUDA.
int set_cuda_error(const char* what, cudaError_t e = cudaErrorUnknown);

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
// A 2-D row-major tensor of `inner` x `outer` elements, `row_stride` elements
// between rows, copied in boxes of box_inner x box_outer, OOB reads as zero.
int encode_tmap_2d(CUtensorMap* map, CUtensorMapDataType dt, int elem_bytes, const void* base,
                   int64_t inner, int64_t outer, int64_t row_stride, uint32_t box_inner,
                   uint32_t box_outer, CUtensorMapSwizzle swizzle);

// 3-D view of a 16-bit [rows x K] row-major tensor as (64 elements, rows,
// K/64 whole k-blocks) with the 128-byte swizzle: a box of box_rows x box_kb
// k-blocks lands in shared memory as box_kb consecutive [box_rows x 128 B]
// blocks, exactly as box_kb 2-D [64 x box_rows] loads would.  Only whole
// k-blocks are addressable (a ragged last k-block needs the 2-D map).
int encode_tmap_kblocks_3d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, int64_t K,
                           int64_t rows, int64_t row_stride, uint32_t box_rows, uint32_t box_kb);

// Generic 3-D tiled map (dims and box innermost first, byte strides of dims
// 1 and 2), OOB reads as zero.
int encode_tmap_3d(CUtensorMap* map, CUtensorMapDataType dt, const void* base,
                   const uint64_t (&dims)[3], const uint64_t (&strides)[2],
                   const uint32_t (&box)[3], CUtensorMapSwizzle swizzle);

int sm_count(int device);
// Bound on every in-kernel wait (FRN_WAIT_TIMEOUT_MS, default 2000 ms).
uint64_t wait_timeout_ns();

int choose_prefill_kernel(int64_t M, int64_t N, int sms);
int run_fused_linear_prefill(const LinearProblem& pr, int kernel, cudaStream_t s);
// SM-pair (cta_group::2) kernel: a pair tile is 256 x (nacc * bn).
struct PairChoice {
  int bn;
  int nacc;
};
// tile64: only tilings whose output tile width is a multiple of 64 columns
// (split outputs store whole 64-column chunks per part).
PairChoice choose_pair_tiling(int64_t M, int64_t N, int64_t K, int pairs, bool tile64 = false);
int run_fused_linear_pair(const LinearProblem& pr, PairChoice c, cudaStream_t s);
// SwiGLU on the pair kernel: pr.w = [gate; up] with pr.N = 2 * inter rows;
// the output has `inter` columns; tiles are 256 x bn output columns.
int choose_swiglu_bn(int64_t M, int64_t inter, int64_t K, int pairs);
int run_fused_swiglu_pair(const LinearProblem& pr, int64_t inter, int bn, cudaStream_t s);
// Decode (M <= 128) swap-AB kernel, `split` CTAs per cluster along K.
int choose_decode_split(int64_t N, int64_t K, int sms);
int run_fused_linear_decode(const LinearProblem& pr, int split, cudaStream_t s);
int run_fused_swiglu_decode(const LinearProblem& pr, int64_t inter, int split, cudaStream_t s);

int run_fused_linear_w8(const W8Problem& pr, cudaStream_t s);
// One or two independent problems of the same dtype in one launch.
int run_fused_linear_w8_group(const W8Problem* prs, int nprob, cudaStream_t s);
int run_quantize_int8(int dtype, const void* w, int64_t N, int64_t K, int64_t ws, void* q,
                      int64_t qs, float* scale, cudaStream_t s);

// Decode-step grouped-query attention (frn_gqa_decode.cu).
struct GqaProblem {
  int dtype;
  const void* q;  // [B, Hq, D]
  const void* k;  // [B, T, Hkv, D]
  const void* v;  // [B, T, Hkv, D]
  void* out;      // [B, Hq, D]
  int64_t B, Hq, Hkv, D, T;
  float scale;
  void* workspace;
  size_t workspace_bytes;
};
size_t gqa_workspace_bytes(int64_t B, int64_t Hq, int64_t D, int64_t S);
int gqa_choose_splits(int64_t B, int64_t Hq, int64_t Hkv, int64_t D, int64_t T, int sms,
                      size_t workspace_bytes);
int run_gqa_decode(const GqaProblem& g, int splits, cudaStream_t s);
// Tensor-core kernel (frn_gqa_decode_mma.cu) for bf16 / fp16, D 64 or 128,
// G <= 8, splits merged inside a cluster (no workspace used); run_gqa_decode
// picks it when it applies.  The split count may come down (never up) to keep
// every CTA resident and the cluster portable (<= 8).
bool gqa_mma_supported(const GqaProblem& g);
int run_gqa_decode_mma(const GqaProblem& g, int splits, cudaStream_t s);
// Static device scratch of the allocation-free GQA entry point.
int gqa_noalloc_scratch(int dev, void** ptr);
size_t gqa_noalloc_scratch_bytes();

int run_rmsnorm_swiglu(int dtype, const void* x, int64_t xs, const void* raw, int64_t rs,
                       void* out, int64_t os, const void* b, int64_t rows, int64_t h,
                       int64_t inter, float eps, int threads, cudaStream_t s);
int run_rmsnorm_normalize(int dtype, const void* x, int64_t xs, void* out, int64_t os,
                          const void* b, int64_t rows, int64_t h, int64_t n, float eps,
                          int threads, cudaStream_t s);

}  // namespace frn
