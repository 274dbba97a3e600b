/*
 * frn_b200.h -- C ABI of the B200 (sm_100a) fused RMSNorm -> Linear library.
 *
 * Every entry point takes plain device pointers, element strides and sizes,
 * runs asynchronously on the given CUDA stream (NULL = legacy default stream)
 * and returns an FRN_* status.  No entry point synchronises the stream.
 * Every call works on the caller's current CUDA device (cudaSetDevice): the
 * pointers and the stream must belong to it.
 * The message of the last failing call on the calling thread is available
 * from frn_last_error().
 *
 * Math (shared by every fused entry point):
 *     inv_rms[m] = rsqrt(sum_k x[m,k]^2 / K + eps)            (fp32)
 *     out[m,n]   = round(inv_rms[m] * sum_k x[m,k] * W[n,k] + b[n])
 * with W the gamma-folded weight W_fused = W * gamma
 * (src/weight_transform.py:69-109 of the reference).  The dot product is
 * accumulated in fp32 on the tcgen05 tensor cores; inv_rms and b are applied
 * to the fp32 accumulator before the single rounding to the output type.
 *
 * Layout rules for the fused entry points: all matrices are row-major with
 * unit stride along K (x, W) and along N (out); row strides are given in
 * elements and must make every row start 16-byte aligned; base pointers must
 * be 16-byte aligned.  A row stride larger than the row length (a strided
 * view such as DeepseekV3's k_pass, row stride 576 for K = 512) is honoured.
 */
#ifndef FRN_B200_H
#define FRN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define FRN_OK                    0
#define FRN_ERR_INVALID_ARGUMENT  1  /* shape / null pointer / rank mistakes  */
#define FRN_ERR_UNSUPPORTED       2  /* dtype or shape the kernel cannot do  */
#define FRN_ERR_MISALIGNED        3  /* pointer or row stride not 16B-legal  */
#define FRN_ERR_WORKSPACE         4  /* workspace missing or too small       */
#define FRN_ERR_CUDA              5  /* CUDA runtime / driver call failed    */
#define FRN_ERR_DEVICE_TIMEOUT    6  /* a bounded in-kernel wait expired     */

/* ---- element types ----------------------------------------------------- */
#define FRN_DTYPE_F32   0
#define FRN_DTYPE_F16   1
#define FRN_DTYPE_BF16  2

/* ---- kernel selection for frn_fused_rmsnorm_linear_ex ------------------ */
#define FRN_KERNEL_AUTO         0  /* DECODE for M <= 128, else PAIR_AUTO     */
#define FRN_KERNEL_TILE_N128    1  /* one SM per 128x128 tile                 */
#define FRN_KERNEL_TILE_N192    2  /* one SM per 128x192 tile                 */
#define FRN_KERNEL_TILE_N256    3  /* one SM per 128x256 tile                 */
#define FRN_KERNEL_DECODE       4  /* swap-AB split-K cluster kernel, M<=128  */
#define FRN_KERNEL_PAIR_N128    5  /* SM pair (cta_group::2) per 256x128 tile */
#define FRN_KERNEL_PAIR_N160    6  /* SM pair per 256x160 tile                */
#define FRN_KERNEL_PAIR_N192    7  /* SM pair per 256x192 tile                */
#define FRN_KERNEL_PAIR_N224    8  /* SM pair per 256x224 tile                */
#define FRN_KERNEL_PAIR_N256    9  /* SM pair per 256x256 tile                */
#define FRN_KERNEL_PAIR_AUTO   10  /* SM pair, tiling chosen by (M, N, K)     */
#define FRN_KERNEL_WIDE_N128   11  /* SM pair, two accumulators: 256x(2*128)  */
#define FRN_KERNEL_WIDE_N192   12  /* SM pair, two accumulators: 256x(2*192)  */
#define FRN_KERNEL_WIDE_N224   13  /* SM pair, two accumulators: 256x(2*224)  */
#define FRN_KERNEL_WIDE_N256   14  /* SM pair, two accumulators: 256x(2*256)  */
#define FRN_KERNEL_WIDE_N176   21  /* SM pair, two accumulators: 256x(2*176)  */

/* Device error-word bits (frn_device_error). */
#define FRN_DEVERR_WAIT_TIMEOUT  0x1u  /* an mbarrier wait ran out            */

/* Version of this ABI; bumped on any signature change. */
int frn_abi_version(void);

/* Message of the last failing call on this thread ("" if none). */
const char* frn_last_error(void);

/*
 * In-place RMSNorm rescale of a precomputed GEMM output:
 *     raw_output[r, c] = round(raw_output[r, c] * inv_rms[r] + b_new[c])
 * inv_rms[r] = rsqrt(sum_k x[r,k]^2 / h + eps).  dtype applies to x,
 * raw_output and b_new alike.  threads_per_row is 256 (the reference's V1)
 * or 512 (V3); the result does not depend on it.
 * Replaces rmsnorm_normalize_cuda / rmsnorm_normalize_512_cuda
 * (reference csrc/denominator_kernel.cu:1947-1989 and :1992-2034, bound in
 * csrc/denominator.cpp:179-193).  Unlike the reference it honours the row
 * stride of x and of raw_output.
 */
int frn_rmsnorm_normalize(int dtype,
                          const void* x, int64_t x_row_stride,
                          void* raw_output, int64_t out_row_stride,
                          const void* b_new,
                          int64_t rows, int64_t h, int64_t out_dim,
                          float eps, int threads_per_row, void* stream);

/*
 * Bytes of device workspace frn_fused_rmsnorm_linear needs for this shape
 * (0 when the chosen kernel needs none).
 */
size_t frn_fused_rmsnorm_linear_workspace_size(int dtype, int64_t M,
                                               int64_t N, int64_t K);

/*
 * Fused RMSNorm -> Linear, one launch:
 *     out[M,N] = round(inv_rms[m] * (x[M,K] . W[N,K]^T) + bias[N])
 * dtype is FRN_DTYPE_BF16 or FRN_DTYPE_F16 (x, W, bias, out share it).
 * bias may be NULL (treated as zeros).  workspace may be NULL when
 * frn_fused_rmsnorm_linear_workspace_size() returned 0.
 * Replaces the pair F.linear(x_2d, W_new) + rmsnorm_normalize(_512)(...)
 * of FusedRMSNormLinearV1/V3.forward (reference src/fused_forward.py:158-167,
 * :182-191) and the functional forms at src/fused_forward.py:316-349.
 */
int frn_fused_rmsnorm_linear(int dtype,
                             const void* x, int64_t M, int64_t K,
                             int64_t x_row_stride,
                             const void* w, int64_t N, int64_t w_row_stride,
                             const void* bias, float eps,
                             void* out, int64_t out_row_stride,
                             void* workspace, size_t workspace_bytes,
                             void* stream);

/* As frn_fused_rmsnorm_linear with an explicit FRN_KERNEL_* choice. */
int frn_fused_rmsnorm_linear_ex(int dtype,
                                const void* x, int64_t M, int64_t K,
                                int64_t x_row_stride,
                                const void* w, int64_t N, int64_t w_row_stride,
                                const void* bias, float eps,
                                void* out, int64_t out_row_stride,
                                void* workspace, size_t workspace_bytes,
                                int kernel, void* stream);

/*
 * Fused RMSNorm -> Linear with int8 weights:
 *     out[M,N] = round(inv_rms[m] * w_scale[n] * (x[M,K] . wq[N,K]^T) + bias[N])
 * dtype (FRN_DTYPE_BF16 / FRN_DTYPE_F16) applies to x, bias and out; wq is
 * int8 row-major (row stride in bytes, a multiple of 16), w_scale fp32 [N]
 * (16-byte aligned).  The int8 bytes are what crosses HBM; they are widened
 * to the x type in shared memory inside the GEMM mainloop.
 * Replaces dequantize_int8 + F.linear(x * bf16(inv_rms), W_deq) of the
 * reference's quantization-aware path (src/benchmark_kimi26_quantized.py:38-39,
 * :102-106), which materialises the bf16 weight on every call.
 */
int frn_fused_rmsnorm_linear_w8(int dtype,
                                const void* x, int64_t M, int64_t K,
                                int64_t x_row_stride,
                                const int8_t* wq, int64_t N, int64_t wq_row_stride,
                                const float* w_scale, const void* bias, float eps,
                                void* out, int64_t out_row_stride, void* stream);

/*
 * One int8-weight problem of frn_fused_rmsnorm_linear_w8_grouped: the
 * arguments of frn_fused_rmsnorm_linear_w8 for one (x, wq) pair, same rules.
 */
typedef struct frn_w8_linear {
  const void* x;
  int64_t M, K, x_row_stride;
  const int8_t* wq;
  int64_t N, wq_row_stride;
  const float* w_scale;
  const void* bias; /* may be NULL */
  void* out;
  int64_t out_row_stride;
} frn_w8_linear;

/*
 * nproblems (1 or 2) independent frn_fused_rmsnorm_linear_w8 problems of one
 * dtype and eps in ONE launch -- e.g. an MLA layer's q_b and kv_b, which read
 * different inputs.  Each SM pair runs its share of both problems' tiles
 * back to back, so one problem's mainloop overlaps the other's last epilogue
 * and the launch's fixed cost is paid once.  That pays off while each
 * problem has at most 256 rows; with more, the two run as consecutive
 * launches.  No output may alias an input of either problem.  Same results
 * (bit for bit) as two frn_fused_rmsnorm_linear_w8 calls.
 * No counterpart in the reference, which launches each projection on its
 * own (src/benchmark_kimi26_quantized.py:102-106).
 */
int frn_fused_rmsnorm_linear_w8_grouped(int dtype, const frn_w8_linear* problems,
                                        int nproblems, float eps, void* stream);

/*
 * Symmetric per-output-channel int8 quantization of a (gamma-folded) weight
 * w[N,K] (dtype fp32 / fp16 / bf16):
 *     scale[n] = max(max_k |w[n,k]|, 1e-8) / 127        (fp32)
 *     q[n,k]   = clamp(round_half_even(w[n,k] / scale[n]), -127, 127)
 * Same numbers as quantize_int8_per_output_channel
 * (reference src/benchmark_kimi26_quantized.py:30-35), on the GPU.
 */
int frn_quantize_int8_per_channel(int dtype, const void* w, int64_t N, int64_t K,
                                  int64_t w_row_stride, int8_t* q, int64_t q_row_stride,
                                  float* scale, void* stream);

/*
 * frn_fused_rmsnorm_linear with the output columns written straight into
 * `nparts` (1..4) separate tensors: part i takes the next part_cols[i]
 * columns (a positive multiple of 8; of 64 when M > 128) and is stored at
 * part_out[i] with row stride part_row_stride[i] elements.  The widths sum to
 * N.  Replaces FusedRMSNormCombinedLinearV1/V3.forward's split + per-part
 * .contiguous() copies (reference src/fused_forward.py:194-251, :222-224).
 */
#define FRN_MAX_PARTS 4
int frn_fused_rmsnorm_linear_split(int dtype, const void* x, int64_t M, int64_t K,
                                   int64_t x_row_stride, const void* w, int64_t N,
                                   int64_t w_row_stride, const void* bias, float eps, int nparts,
                                   const int64_t* part_cols, void* const* part_out,
                                   const int64_t* part_row_stride, void* stream);

/*
 * RMSNorm + SwiGLU epilogue of a precomputed [gate | up] GEMM output
 * raw_output[rows, 2*intermediate] (raw = x . W_combined^T):
 *     g = raw[r, c] * inv_rms[r] + b_new[c]
 *     u = raw[r, intermediate + c] * inv_rms[r] + b_new[intermediate + c]
 *     output[r, c] = round(g / (1 + exp(-g)) * u)       for c < intermediate
 * inv_rms as in frn_rmsnorm_normalize; b_new has 2*intermediate entries.
 * Replaces rmsnorm_swiglu_cuda / rmsnorm_swiglu_512_cuda (reference
 * csrc/denominator_kernel.cu:2037-2134, bound in csrc/denominator.cpp:152-213)
 * and honours all three row strides.
 */
int frn_rmsnorm_swiglu(int dtype, const void* x, int64_t x_row_stride, const void* raw_output,
                       int64_t raw_row_stride, void* output, int64_t out_row_stride,
                       const void* b_new, int64_t rows, int64_t h, int64_t intermediate,
                       float eps, int threads_per_row, void* stream);

/*
 * Fused RMSNorm -> [gate | up] projection -> SwiGLU in one kernel:
 *     acc_g[m, c] = sum_k x[m,k] * Wc[c, k]
 *     acc_u[m, c] = sum_k x[m,k] * Wc[intermediate + c, k]
 *     out[m, c] = round(silu(acc_g * inv_rms[m] + b[c]) *
 *                       (acc_u * inv_rms[m] + b[intermediate + c]))
 * w_combined is the gamma-folded [gate; up] weight (2*intermediate rows of K),
 * bias has 2*intermediate entries or is NULL; the [M, 2*intermediate] GEMM
 * output is never written to memory.  bf16 / fp16; same layout rules as
 * frn_fused_rmsnorm_linear with N = 2*intermediate (intermediate % 8 == 0).
 * Replaces FusedRMSNormSwiGLUV1/V3.forward (reference
 * src/fused_forward.py:254-313): F.linear(x, W_combined) followed by
 * rmsnorm_swiglu(_512).
 */
int frn_fused_rmsnorm_swiglu(int dtype, const void* x, int64_t M, int64_t K,
                             int64_t x_row_stride, const void* w_combined, int64_t intermediate,
                             int64_t w_row_stride, const void* bias, float eps, void* out,
                             int64_t out_row_stride, void* stream);

/*
 * Decode-step grouped-query attention (one query token per sequence):
 *     out[b, h, :] = softmax_t(scale * q[b, h, :] . K[b, t, h/G, :]) @ V[b, :, h/G, :]
 * q [batch, num_q_heads, head_dim], k_cache / v_cache [batch, context_len,
 * num_kv_heads, head_dim], out [batch, num_q_heads, head_dim], all contiguous
 * and of `dtype` (fp32 / fp16 / bf16); head_dim 64 or 128; G = num_q_heads /
 * num_kv_heads <= 8.  bf16 / fp16 run on the tensor-core kernel, which splits
 * the context over a thread-block cluster and merges the splits on chip: it
 * never reads the workspace.  fp32 runs the CUDA-core kernel, whose context
 * split writes partials to `workspace` (frn_gqa_decode_workspace_size bytes)
 * for a second merge launch; with no workspace each (batch, KV head) of an
 * fp32 call is one CTA.  Replaces gqa_decode_v2_cuda / gqa_decode_v3_cuda
 * (reference csrc/gqa_attention_kernel.cu:357-470, bound in
 * csrc/gqa_attention.cpp:45-60), on the caller's stream.
 *
 * frn_gqa_decode_workspace_size returns what the fp32 split path needs for
 * the shape (an upper bound for every dtype; bf16 / fp16 calls may pass no
 * workspace at all).  With G <= 8 and head_dim <= 128 the split rule keeps it
 * at or below 3 * SMs * G * (head_dim + 2) * 4 bytes (1.85 MB on a 148-SM
 * B200).
 */
size_t frn_gqa_decode_workspace_size(int64_t batch, int64_t num_q_heads, int64_t num_kv_heads,
                                     int64_t head_dim, int64_t context_len);
int frn_gqa_decode_attention(int dtype, const void* q, const void* k_cache, const void* v_cache,
                             void* out, int64_t batch, int64_t num_q_heads,
                             int64_t num_kv_heads, int64_t head_dim, int64_t context_len,
                             float scale, void* workspace, size_t workspace_bytes,
                             void* stream);

/*
 * frn_gqa_decode_attention without a workspace argument and without any
 * allocation: for callers that cannot allocate device memory at call time --
 * hosts whose device memory is wholly reserved up front by their own
 * allocator or memory pool, or that forbid cudaMalloc/cudaFree on their
 * decode path -- and so cannot hand the kernel the workspace its context
 * split needs.  bf16 / fp16 calls need no scratch (the tensor-core kernel
 * merges its splits on chip).  An fp32 call parks its split partials in a
 * fixed 2 MiB scratch array inside this library (one per device; its device
 * address is looked up on the first fp32 call on that device, so make that
 * first call before any stream capture).  An fp32 shape needing more scratch
 * than that is rejected with FRN_ERR_UNSUPPORTED (on a 148-SM B200 no valid
 * shape does, see frn_gqa_decode_workspace_size).  Every fp32 call shares
 * that one array, so fp32 calls whose work overlaps on the GPU (different
 * streams, or no ordering between them) race and corrupt each other's
 * results; issue them in order on one stream.  Nothing in the scratch has to
 * start at zero.  Same results as frn_gqa_decode_attention given its full
 * workspace.
 * No counterpart in the reference.
 */
int frn_gqa_decode_attention_noalloc(int dtype, const void* q, const void* k_cache,
                                     const void* v_cache, void* out, int64_t batch,
                                     int64_t num_q_heads, int64_t num_kv_heads,
                                     int64_t head_dim, int64_t context_len, float scale,
                                     void* stream);

/*
 * Reads (and optionally clears) the device error word of `device`, which
 * kernels set when a bounded wait expires instead of hanging.  Synchronous
 * with respect to the device's legacy default stream.
 */
int frn_device_error(int device, uint32_t* flags, int clear);

/*
 * Failure-detection self-test: launches a one-thread kernel on `stream` that
 * waits on an mbarrier nothing ever arrives at, using the bounded wait of
 * every pipeline role in this library.  After timeout_ms (1..10000) the wait
 * gives up, sets FRN_DEVERR_WAIT_TIMEOUT in the device error word and the
 * kernel returns normally (no trap; the context stays usable).  Read the word
 * with frn_device_error.  No counterpart in the reference, whose launchers
 * have no device-side failure reporting.
 */
int frn_selftest_wait_timeout(int timeout_ms, void* stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif /* FRN_B200_H */
