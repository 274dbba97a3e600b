// frn_capi.cu -- the extern "C" boundary declared in include/frn_b200.h:
// argument validation (the reference's TORCH_CHECKs plus the alignment and
// stride rules TMA needs), kernel choice, and error reporting.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "frn_internal.h"
#include "frn_ptx.cuh"

namespace frn {

__device__ uint32_t g_frn_device_error = 0u;

static thread_local char t_last_error[512] = {0};

// Failure-detection self-test: one thread waits, with the same bounded
// mbarrier wait every pipeline role uses, on a barrier nothing arrives at.
// The wait gives up after timeout_ns, ORs kDevErrWaitTimeout into the device
// error word and the kernel returns; no trap, the context stays usable.
__global__ void selftest_wait_timeout_kernel(uint64_t timeout_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t abort_flag;
  if (threadIdx.x != 0) return;
  abort_flag = 0u;
  mbar_init(&bar, 1);
  fence_mbarrier_init();
  mbar_wait(&bar, 0, &abort_flag, timeout_ns);
}

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int set_cuda_error(const char* what, cudaError_t e) {
  return set_error(FRN_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, []() {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int encode_tmap_2d(CUtensorMap* map, CUtensorMapDataType dt, int elem_bytes, const void* base,
                   int64_t inner, int64_t outer, int64_t row_stride, uint32_t box_inner,
                   uint32_t box_outer, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn enc = get_encode_tiled();
  if (!enc) return set_error(FRN_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_stride) * elem_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(FRN_ERR_INVALID_ARGUMENT,
                     "cuTensorMapEncodeTiled failed (%d) for a %lld x %lld tensor, row stride "
                     "%lld elements",
                     static_cast<int>(r), static_cast<long long>(outer),
                     static_cast<long long>(inner), static_cast<long long>(row_stride));
  return 0;
}

int encode_tmap_kblocks_3d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, int64_t K,
                           int64_t rows, int64_t row_stride, uint32_t box_rows, uint32_t box_kb) {
  EncodeTiledFn enc = get_encode_tiled();
  if (!enc) return set_error(FRN_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  const int64_t full = K / 64;
  const cuuint64_t dims[3] = {64, static_cast<cuuint64_t>(rows),
                              static_cast<cuuint64_t>(full > 0 ? full : 1)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(row_stride) * 2, 128};
  const cuuint32_t box[3] = {64, box_rows,
                             static_cast<cuuint32_t>(full > 0 && full < box_kb ? full : box_kb)};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(FRN_ERR_INVALID_ARGUMENT,
                     "cuTensorMapEncodeTiled failed (%d) for the k-block view of a %lld x %lld "
                     "tensor",
                     static_cast<int>(r), static_cast<long long>(rows), static_cast<long long>(K));
  return 0;
}

int encode_tmap_3d(CUtensorMap* map, CUtensorMapDataType dt, const void* base,
                   const uint64_t (&dims)[3], const uint64_t (&strides)[2],
                   const uint32_t (&box)[3], CUtensorMapSwizzle swizzle) {
  EncodeTiledFn enc = get_encode_tiled();
  if (!enc) return set_error(FRN_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  const cuuint64_t d[3] = {dims[0], dims[1], dims[2]};
  const cuuint64_t st[2] = {strides[0], strides[1]};
  const cuuint32_t bx[3] = {box[0], box[1], box[2]};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, dt, 3, const_cast<void*>(base), d, st, bx, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(FRN_ERR_INVALID_ARGUMENT, "cuTensorMapEncodeTiled failed (%d) for a 3-D view",
                     static_cast<int>(r));
  return 0;
}

int sm_count(int device) {
  static int cache[kMaxDevices] = {0};
  if (device >= 0 && device < kMaxDevices && cache[device] > 0) return cache[device];
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n <= 0)
    n = 148;
  if (device >= 0 && device < kMaxDevices) cache[device] = n;
  return n;
}

uint64_t wait_timeout_ns() {
  static uint64_t v = 0;
  if (v == 0) {
    const char* s = std::getenv("FRN_WAIT_TIMEOUT_MS");
    long long ms = s ? std::atoll(s) : 0;
    if (ms <= 0) ms = 2000;
    v = static_cast<uint64_t>(ms) * 1000000ull;
  }
  return v;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

static int elem_bytes(int dtype) {
  return dtype == FRN_DTYPE_F32 ? 4 : 2;
}

static int validate_linear(const LinearProblem& p) {
  if (p.dtype != FRN_DTYPE_BF16 && p.dtype != FRN_DTYPE_F16)
    return set_error(FRN_ERR_UNSUPPORTED,
                     "fused RMSNorm+Linear supports bf16 and fp16 only (dtype %d)", p.dtype);
  if (p.M < 0 || p.N <= 0 || p.K <= 0)
    return set_error(FRN_ERR_INVALID_ARGUMENT, "bad shape M=%lld N=%lld K=%lld",
                     (long long)p.M, (long long)p.N, (long long)p.K);
  if (p.M > 0x7fffffffLL || p.N > 0x7fffffffLL || p.K > 0x7fffffffLL)
    return set_error(FRN_ERR_UNSUPPORTED, "dimension exceeds 2^31-1");
  if (p.M > 0 && (!p.x || !p.w || !p.out))
    return set_error(FRN_ERR_INVALID_ARGUMENT, "x, W and out must be non-null");
  if (p.x_row_stride < p.K || p.w_row_stride < p.K || p.out_row_stride < p.N)
    return set_error(FRN_ERR_INVALID_ARGUMENT,
                     "row strides must be >= row lengths (x %lld/%lld, W %lld/%lld, out %lld/%lld)",
                     (long long)p.x_row_stride, (long long)p.K, (long long)p.w_row_stride,
                     (long long)p.K, (long long)p.out_row_stride, (long long)p.N);
  if (p.K % 8 || p.N % 8)
    return set_error(FRN_ERR_MISALIGNED,
                     "K (%lld) and N (%lld) must be multiples of 8 (16-byte rows for TMA)",
                     (long long)p.K, (long long)p.N);
  if (p.x_row_stride % 8 || p.w_row_stride % 8 || p.out_row_stride % 8)
    return set_error(FRN_ERR_MISALIGNED, "row strides must be multiples of 8 elements (16 bytes)");
  if (!aligned16(p.x) || !aligned16(p.w) || !aligned16(p.out) ||
      (p.bias && !aligned16(p.bias)))
    return set_error(FRN_ERR_MISALIGNED, "x, W, out and bias must be 16-byte aligned");
  return 0;
}

}  // namespace frn

using namespace frn;

extern "C" {

int frn_abi_version(void) { return 1; }

const char* frn_last_error(void) { return t_last_error; }

int frn_rmsnorm_normalize(int dtype, const void* x, int64_t x_row_stride, void* raw_output,
                          int64_t out_row_stride, const void* b_new, int64_t rows, int64_t h,
                          int64_t out_dim, float eps, int threads_per_row, void* stream) {
  if (dtype != FRN_DTYPE_F32 && dtype != FRN_DTYPE_F16 && dtype != FRN_DTYPE_BF16)
    return set_error(FRN_ERR_UNSUPPORTED,
                     "Unsupported dtype for RMSNorm normalize: only fp32, fp16, bf16 supported");
  if (rows < 0 || h <= 0 || out_dim < 0)
    return set_error(FRN_ERR_INVALID_ARGUMENT, "bad shape rows=%lld h=%lld out_dim=%lld",
                     (long long)rows, (long long)h, (long long)out_dim);
  if (threads_per_row != 256 && threads_per_row != 512)
    return set_error(FRN_ERR_INVALID_ARGUMENT, "threads_per_row must be 256 or 512");
  if (rows == 0 || out_dim == 0) return FRN_OK;
  if (!x || !raw_output || !b_new)
    return set_error(FRN_ERR_INVALID_ARGUMENT, "x, raw_output and b_new must be non-null");
  if (x_row_stride < h || out_row_stride < out_dim)
    return set_error(FRN_ERR_INVALID_ARGUMENT, "row strides must be >= row lengths");
  if (rows > 0x7fffffffLL || h > 0x7fffffffLL || out_dim > 0x7fffffffLL)
    return set_error(FRN_ERR_UNSUPPORTED, "dimension exceeds 2^31-1");
  (void)elem_bytes;
  return run_rmsnorm_normalize(dtype, x, x_row_stride, raw_output, out_row_stride, b_new, rows, h,
                               out_dim, eps, threads_per_row,
                               static_cast<cudaStream_t>(stream));
}

int frn_rmsnorm_swiglu(int dtype, const void* x, int64_t x_row_stride, const void* raw_output,
                       int64_t raw_row_stride, void* output, int64_t out_row_stride,
                       const void* b_new, int64_t rows, int64_t h, int64_t intermediate,
                       float eps, int threads_per_row, void* stream) {
  if (dtype != FRN_DTYPE_F32 && dtype != FRN_DTYPE_F16 && dtype != FRN_DTYPE_BF16)
    return set_error(FRN_ERR_UNSUPPORTED,
                     "Unsupported dtype for RMSNorm SwiGLU: only fp32, fp16, bf16 supported");
  if (rows < 0 || h <= 0 || intermediate < 0)
    return set_error(FRN_ERR_INVALID_ARGUMENT, "bad shape rows=%lld h=%lld intermediate=%lld",
                     (long long)rows, (long long)h, (long long)intermediate);
  if (threads_per_row != 256 && threads_per_row != 512)
    return set_error(FRN_ERR_INVALID_ARGUMENT, "threads_per_row must be 256 or 512");
  if (rows == 0 || intermediate == 0) return FRN_OK;
  if (!x || !raw_output || !output || !b_new)
    return set_error(FRN_ERR_INVALID_ARGUMENT, "x, raw_output, output and b_new must be non-null");
  if (x_row_stride < h || raw_row_stride < 2 * intermediate || out_row_stride < intermediate)
    return set_error(FRN_ERR_INVALID_ARGUMENT, "row strides must be >= row lengths");
  if (rows > 0x7fffffffLL || h > 0x7fffffffLL || 2 * intermediate > 0x7fffffffLL)
    return set_error(FRN_ERR_UNSUPPORTED, "dimension exceeds 2^31-1");
  return run_rmsnorm_swiglu(dtype, x, x_row_stride, raw_output, raw_row_stride, output,
                            out_row_stride, b_new, rows, h, intermediate, eps, threads_per_row,
                            static_cast<cudaStream_t>(stream));
}

int frn_fused_rmsnorm_swiglu(int dtype, const void* x, int64_t M, int64_t K,
                             int64_t x_row_stride, const void* w_combined, int64_t intermediate,
                             int64_t w_row_stride, const void* bias, float eps, void* out,
                             int64_t out_row_stride, void* stream) {
  if (intermediate <= 0)
    return set_error(FRN_ERR_INVALID_ARGUMENT, "bad intermediate size %lld",
                     (long long)intermediate);
  if (out_row_stride < intermediate)
    return set_error(FRN_ERR_INVALID_ARGUMENT, "out row stride %lld < intermediate %lld",
                     (long long)out_row_stride, (long long)intermediate);
  // Validated as the [M, 2*intermediate] linear over W_combined; the output
  // stride is checked against its own width above.
  LinearProblem p{dtype, x, M, K, x_row_stride, w_combined, 2 * intermediate, w_row_stride,
                  bias, eps, out, 2 * intermediate, nullptr, 0};
  int rc = validate_linear(p);
  if (rc) return rc;
  if (out_row_stride % 8)
    return set_error(FRN_ERR_MISALIGNED, "row strides must be multiples of 8 elements (16 bytes)");
  p.out_row_stride = out_row_stride;
  if (M == 0) return FRN_OK;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return set_cuda_error("cudaGetDevice");
  const int sms = sm_count(dev);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (M <= 128)
    return run_fused_swiglu_decode(p, intermediate, choose_decode_split(2 * intermediate, K, sms),
                                   s);
  return run_fused_swiglu_pair(p, intermediate, choose_swiglu_bn(M, intermediate, K, sms / 2), s);
}

static int validate_gqa(int dtype, int64_t B, int64_t Hq, int64_t Hkv, int64_t D, int64_t T) {
  if (dtype != FRN_DTYPE_F32 && dtype != FRN_DTYPE_F16 && dtype != FRN_DTYPE_BF16)
    return set_error(FRN_ERR_UNSUPPORTED, "GQA decode supports fp32, fp16 and bf16");
  if (B < 0 || Hq <= 0 || Hkv <= 0 || T <= 0)
    return set_error(FRN_ERR_INVALID_ARGUMENT,
                     "bad shape batch=%lld q_heads=%lld kv_heads=%lld context=%lld",
                     (long long)B, (long long)Hq, (long long)Hkv, (long long)T);
  if (D != 64 && D != 128)
    return set_error(FRN_ERR_UNSUPPORTED, "head_dim must be 64 or 128 (got %lld)", (long long)D);
  if (Hq % Hkv || Hq / Hkv > 8)
    return set_error(FRN_ERR_UNSUPPORTED,
                     "num_q_heads must be a multiple of num_kv_heads with a group of at most 8");
  if (B > 65535 || Hkv > 0x7fffffffLL || T > 0x7fffffffLL || B * T * Hkv * D > (int64_t(1) << 40))
    return set_error(FRN_ERR_UNSUPPORTED, "GQA decode dimensions too large");
  return 0;
}

size_t frn_gqa_decode_workspace_size(int64_t batch, int64_t num_q_heads, int64_t num_kv_heads,
                                     int64_t head_dim, int64_t context_len) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
  const int S = gqa_choose_splits(batch, num_q_heads, num_kv_heads, head_dim, context_len,
                                  sm_count(dev), static_cast<size_t>(-1));
  return gqa_workspace_bytes(batch, num_q_heads, head_dim, S);
}

int frn_gqa_decode_attention(int dtype, const void* q, const void* k_cache, const void* v_cache,
                             void* out, int64_t batch, int64_t num_q_heads,
                             int64_t num_kv_heads, int64_t head_dim, int64_t context_len,
                             float scale, void* workspace, size_t workspace_bytes,
                             void* stream) {
  int rc = validate_gqa(dtype, batch, num_q_heads, num_kv_heads, head_dim, context_len);
  if (rc) return rc;
  if (batch == 0) return FRN_OK;
  if (!q || !k_cache || !v_cache || !out)
    return set_error(FRN_ERR_INVALID_ARGUMENT, "q, k_cache, v_cache and out must be non-null");
  if (!aligned16(q) || !aligned16(k_cache) || !aligned16(v_cache) || !aligned16(out) ||
      (workspace && !aligned16(workspace)))
    return set_error(FRN_ERR_MISALIGNED, "q, caches, out and workspace must be 16-byte aligned");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return set_cuda_error("cudaGetDevice");
  const size_t ws_bytes = workspace ? workspace_bytes : 0;
  GqaProblem g{dtype, q, k_cache, v_cache, out, batch, num_q_heads, num_kv_heads, head_dim,
               context_len, scale, workspace, ws_bytes};
  // The tensor-core kernel merges its splits inside a cluster and never
  // touches the workspace, so its split count is not bounded by it.
  const int S = gqa_choose_splits(batch, num_q_heads, num_kv_heads, head_dim, context_len,
                                  sm_count(dev),
                                  gqa_mma_supported(g) ? static_cast<size_t>(-1) : ws_bytes);
  return run_gqa_decode(g, S, static_cast<cudaStream_t>(stream));
}

int frn_gqa_decode_attention_noalloc(int dtype, const void* q, const void* k_cache,
                                     const void* v_cache, void* out, int64_t batch,
                                     int64_t num_q_heads, int64_t num_kv_heads,
                                     int64_t head_dim, int64_t context_len, float scale,
                                     void* stream) {
  int rc = validate_gqa(dtype, batch, num_q_heads, num_kv_heads, head_dim, context_len);
  if (rc) return rc;
  if (batch == 0) return FRN_OK;
  if (!q || !k_cache || !v_cache || !out)
    return set_error(FRN_ERR_INVALID_ARGUMENT, "q, k_cache, v_cache and out must be non-null");
  if (!aligned16(q) || !aligned16(k_cache) || !aligned16(v_cache) || !aligned16(out))
    return set_error(FRN_ERR_MISALIGNED, "q, caches and out must be 16-byte aligned");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return set_cuda_error("cudaGetDevice");
  // Same split count (hence the same result) as frn_gqa_decode_attention
  // given its full workspace.
  const int S = gqa_choose_splits(batch, num_q_heads, num_kv_heads, head_dim, context_len,
                                  sm_count(dev), static_cast<size_t>(-1));
  GqaProblem g{dtype, q, k_cache, v_cache, out, batch, num_q_heads, num_kv_heads, head_dim,
               context_len, scale, nullptr, 0};
  // bf16 / fp16 shapes go to the tensor-core kernel, which merges its splits
  // through cluster shared memory and needs no scratch at all; only the
  // CUDA-core split + merge path (fp32) parks partials in the static array.
  if (gqa_mma_supported(g)) return run_gqa_decode(g, S, static_cast<cudaStream_t>(stream));
  const size_t need = gqa_workspace_bytes(batch, num_q_heads, head_dim, S);
  if (need > gqa_noalloc_scratch_bytes())
    return set_error(FRN_ERR_UNSUPPORTED,
                     "GQA decode needs %zu bytes of scratch for this shape; the static scratch "
                     "holds %zu (use frn_gqa_decode_attention with a workspace)",
                     need, gqa_noalloc_scratch_bytes());
  if (need > 0) {
    rc = gqa_noalloc_scratch(dev, &g.workspace);
    if (rc) return rc;
    g.workspace_bytes = need;
  }
  return run_gqa_decode(g, S, static_cast<cudaStream_t>(stream));
}

size_t frn_fused_rmsnorm_linear_workspace_size(int dtype, int64_t M, int64_t N, int64_t K) {
  (void)dtype; (void)M; (void)N; (void)K;
  return 0;
}

int frn_fused_rmsnorm_linear_ex(int dtype, const void* x, int64_t M, int64_t K,
                                int64_t x_row_stride, const void* w, int64_t N,
                                int64_t w_row_stride, const void* bias, float eps, void* out,
                                int64_t out_row_stride, void* workspace, size_t workspace_bytes,
                                int kernel, void* stream) {
  LinearProblem p{dtype, x, M, K, x_row_stride, w, N, w_row_stride, bias, eps, out,
                  out_row_stride, workspace, workspace_bytes};
  int rc = validate_linear(p);
  if (rc) return rc;
  if (M == 0) return FRN_OK;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return set_cuda_error("cudaGetDevice");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int sms = sm_count(dev);
  if (kernel == FRN_KERNEL_AUTO) kernel = (M <= 128) ? FRN_KERNEL_DECODE : FRN_KERNEL_PAIR_AUTO;
  if (kernel == FRN_KERNEL_PAIR_AUTO)
    return run_fused_linear_pair(p, choose_pair_tiling(M, N, K, sms / 2), s);
  if (kernel >= FRN_KERNEL_TILE_N128 && kernel <= FRN_KERNEL_TILE_N256)
    return run_fused_linear_prefill(p, kernel, s);
  if (kernel >= FRN_KERNEL_PAIR_N128 && kernel <= FRN_KERNEL_PAIR_N256) {
    static const int bns[5] = {128, 160, 192, 224, 256};
    return run_fused_linear_pair(p, PairChoice{bns[kernel - FRN_KERNEL_PAIR_N128], 1}, s);
  }
  if (kernel >= FRN_KERNEL_WIDE_N128 && kernel <= FRN_KERNEL_WIDE_N256) {
    static const int bns[4] = {128, 192, 224, 256};
    return run_fused_linear_pair(p, PairChoice{bns[kernel - FRN_KERNEL_WIDE_N128], 2}, s);
  }
  if (kernel == FRN_KERNEL_WIDE_N176) return run_fused_linear_pair(p, PairChoice{176, 2}, s);
  if (kernel == FRN_KERNEL_DECODE) {
    if (M > 128)
      return set_error(FRN_ERR_UNSUPPORTED, "the decode kernel takes M <= 128 (got %lld)",
                       (long long)M);
    return run_fused_linear_decode(p, choose_decode_split(N, K, sms), s);
  }
  return set_error(FRN_ERR_UNSUPPORTED, "kernel id %d not available", kernel);
}

int frn_fused_rmsnorm_linear_split(int dtype, const void* x, int64_t M, int64_t K,
                                   int64_t x_row_stride, const void* w, int64_t N,
                                   int64_t w_row_stride, const void* bias, float eps, int nparts,
                                   const int64_t* part_cols, void* const* part_out,
                                   const int64_t* part_row_stride, void* stream) {
  if (nparts < 1 || nparts > kMaxParts)
    return set_error(FRN_ERR_INVALID_ARGUMENT, "nparts must be 1..%d (got %d)", kMaxParts,
                     nparts);
  if (!part_cols || !part_out || !part_row_stride)
    return set_error(FRN_ERR_INVALID_ARGUMENT, "part arrays must be non-null");
  OutParts parts;
  parts.n = nparts;
  int64_t c0 = 0;
  bool all64 = true;
  for (int i = 0; i < nparts; ++i) {
    if (part_cols[i] <= 0 || part_cols[i] % 8)
      return set_error(FRN_ERR_MISALIGNED, "part %d width %lld must be a positive multiple of 8",
                       i, (long long)part_cols[i]);
    if (part_row_stride[i] < part_cols[i] || part_row_stride[i] % 8)
      return set_error(FRN_ERR_MISALIGNED,
                       "part %d row stride %lld must be >= its width and a multiple of 8", i,
                       (long long)part_row_stride[i]);
    if (M > 0 && (!part_out[i] || !aligned16(part_out[i])))
      return set_error(FRN_ERR_MISALIGNED, "part %d output must be non-null and 16-byte aligned",
                       i);
    all64 = all64 && (part_cols[i] % 64 == 0);
    parts.col0[i] = c0;
    parts.cols[i] = part_cols[i];
    parts.out[i] = part_out[i];
    parts.stride[i] = part_row_stride[i];
    c0 += part_cols[i];
  }
  if (c0 != N)
    return set_error(FRN_ERR_INVALID_ARGUMENT, "part widths sum to %lld, N is %lld",
                     (long long)c0, (long long)N);
  // Validated as a plain [M, N] linear (the first part stands in for out).
  LinearProblem p{dtype, x, M, K, x_row_stride, w, N, w_row_stride, bias, eps,
                  part_out[0], N, nullptr, 0};
  int rc = validate_linear(p);
  if (rc) return rc;
  p.out_row_stride = part_row_stride[0];
  p.parts = &parts;
  if (M == 0) return FRN_OK;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return set_cuda_error("cudaGetDevice");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int sms = sm_count(dev);
  if (M <= 128) return run_fused_linear_decode(p, choose_decode_split(N, K, sms), s);
  if (!all64 && nparts > 1)
    return set_error(FRN_ERR_UNSUPPORTED,
                     "for M > 128 the split parts must be multiples of 64 columns");
  return run_fused_linear_pair(p, choose_pair_tiling(M, N, K, sms / 2, nparts > 1), s);
}

int frn_fused_rmsnorm_linear(int dtype, const void* x, int64_t M, int64_t K, int64_t x_row_stride,
                             const void* w, int64_t N, int64_t w_row_stride, const void* bias,
                             float eps, void* out, int64_t out_row_stride, void* workspace,
                             size_t workspace_bytes, void* stream) {
  return frn_fused_rmsnorm_linear_ex(dtype, x, M, K, x_row_stride, w, N, w_row_stride, bias, eps,
                                     out, out_row_stride, workspace, workspace_bytes,
                                     FRN_KERNEL_AUTO, stream);
}

// Argument checks of one int8-weight problem (both entry points).
static int validate_w8(int dtype, const void* x, int64_t M, int64_t K, int64_t x_row_stride,
                       const int8_t* wq, int64_t N, int64_t wq_row_stride, const float* w_scale,
                       const void* bias, const void* out, int64_t out_row_stride) {
  if (dtype != FRN_DTYPE_BF16 && dtype != FRN_DTYPE_F16)
    return set_error(FRN_ERR_UNSUPPORTED, "int8-weight RMSNorm+Linear takes bf16 or fp16 x");
  if (M < 0 || N <= 0 || K <= 0)
    return set_error(FRN_ERR_INVALID_ARGUMENT, "bad shape M=%lld N=%lld K=%lld", (long long)M,
                     (long long)N, (long long)K);
  if (M > 0x7fffffffLL || N > 0x7fffffffLL || K > 0x7fffffffLL)
    return set_error(FRN_ERR_UNSUPPORTED, "dimension exceeds 2^31-1");
  if (M == 0) return FRN_OK;
  if (!x || !wq || !w_scale || !out)
    return set_error(FRN_ERR_INVALID_ARGUMENT, "x, wq, w_scale and out must be non-null");
  if (x_row_stride < K || wq_row_stride < K || out_row_stride < N)
    return set_error(FRN_ERR_INVALID_ARGUMENT, "row strides must be >= row lengths");
  if (K % 16 || N % 8 || x_row_stride % 8 || out_row_stride % 8 || wq_row_stride % 16)
    return set_error(FRN_ERR_MISALIGNED,
                     "K must be a multiple of 16, N of 8; x/out row strides multiples of 8 "
                     "elements, wq row stride a multiple of 16 bytes");
  if (!aligned16(x) || !aligned16(wq) || !aligned16(w_scale) || !aligned16(out) ||
      (bias && !aligned16(bias)))
    return set_error(FRN_ERR_MISALIGNED, "x, wq, w_scale, bias and out must be 16-byte aligned");
  return FRN_OK;
}

int frn_fused_rmsnorm_linear_w8(int dtype, const void* x, int64_t M, int64_t K,
                                int64_t x_row_stride, const int8_t* wq, int64_t N,
                                int64_t wq_row_stride, const float* w_scale, const void* bias,
                                float eps, void* out, int64_t out_row_stride, void* stream) {
  const int rc = validate_w8(dtype, x, M, K, x_row_stride, wq, N, wq_row_stride, w_scale, bias,
                             out, out_row_stride);
  if (rc || M == 0) return rc;
  W8Problem p{dtype, x, M, K, x_row_stride, wq, N, wq_row_stride, w_scale, bias, eps, out,
              out_row_stride};
  return run_fused_linear_w8(p, static_cast<cudaStream_t>(stream));
}

int frn_fused_rmsnorm_linear_w8_grouped(int dtype, const frn_w8_linear* problems,
                                        int nproblems, float eps, void* stream) {
  if (!problems || nproblems < 1 || nproblems > 2)
    return set_error(FRN_ERR_INVALID_ARGUMENT, "grouped int8 call takes 1 or 2 problems (got %d)",
                     nproblems);
  W8Problem ps[2];
  int n = 0;
  for (int j = 0; j < nproblems; ++j) {
    const frn_w8_linear& q = problems[j];
    const int rc = validate_w8(dtype, q.x, q.M, q.K, q.x_row_stride, q.wq, q.N, q.wq_row_stride,
                               q.w_scale, q.bias, q.out, q.out_row_stride);
    if (rc) return rc;
    if (q.M == 0) continue;  // nothing to do for this one
    ps[n++] = W8Problem{dtype, q.x, q.M, q.K, q.x_row_stride, q.wq, q.N, q.wq_row_stride,
                        q.w_scale, q.bias, eps, q.out, q.out_row_stride};
  }
  if (n == 0) return FRN_OK;
  return run_fused_linear_w8_group(ps, n, static_cast<cudaStream_t>(stream));
}

int frn_quantize_int8_per_channel(int dtype, const void* w, int64_t N, int64_t K,
                                  int64_t w_row_stride, int8_t* q, int64_t q_row_stride,
                                  float* scale, void* stream) {
  if (dtype != FRN_DTYPE_F32 && dtype != FRN_DTYPE_F16 && dtype != FRN_DTYPE_BF16)
    return set_error(FRN_ERR_UNSUPPORTED, "quantize: weight dtype must be fp32, fp16 or bf16");
  if (N < 0 || K <= 0 || w_row_stride < K || q_row_stride < K)
    return set_error(FRN_ERR_INVALID_ARGUMENT, "quantize: bad shape or strides");
  if (N == 0) return FRN_OK;
  if (!w || !q || !scale)
    return set_error(FRN_ERR_INVALID_ARGUMENT, "quantize: w, q and scale must be non-null");
  if (N > 0x7fffffffLL || K > 0x7fffffffLL)
    return set_error(FRN_ERR_UNSUPPORTED, "dimension exceeds 2^31-1");
  return run_quantize_int8(dtype, w, N, K, w_row_stride, q, q_row_stride, scale,
                           static_cast<cudaStream_t>(stream));
}

int frn_selftest_wait_timeout(int timeout_ms, void* stream) {
  if (timeout_ms <= 0 || timeout_ms > 10000)
    return set_error(FRN_ERR_INVALID_ARGUMENT, "timeout_ms must be in 1..10000");
  selftest_wait_timeout_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<uint64_t>(timeout_ms) * 1000000ull);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error("launch selftest_wait_timeout", e);
  return FRN_OK;
}

int frn_device_error(int device, uint32_t* flags, int clear) {
  if (!flags) return set_error(FRN_ERR_INVALID_ARGUMENT, "flags must be non-null");
  int prev = 0;
  if (cudaGetDevice(&prev) != cudaSuccess) return set_cuda_error("cudaGetDevice");
  if (device != prev && cudaSetDevice(device) != cudaSuccess)
    return set_cuda_error("cudaSetDevice");
  cudaError_t e = cudaMemcpyFromSymbol(flags, g_frn_device_error, sizeof(uint32_t));
  if (e == cudaSuccess && clear) {
    const uint32_t zero = 0;
    e = cudaMemcpyToSymbol(g_frn_device_error, &zero, sizeof(uint32_t));
  }
  if (device != prev) cudaSetDevice(prev);
  if (e != cudaSuccess) return set_cuda_error("reading the device error word", e);
  return FRN_OK;
}

}  // extern "C"
