// frn_ptx.cuh -- thin inline-PTX wrappers for sm_100a: mbarriers with bounded
// waits, TMA tile loads/stores, and the tcgen05 (TMEM + UMMA) instructions the
// fused kernels use.  Nothing here allocates or launches.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace frn {

// Device-wide error word (see frn_device_error in include/frn_b200.h).  A
// kernel whose bounded wait expires ORs a bit in here and winds down instead
// of hanging the GPU.
extern __device__ uint32_t g_frn_device_error;

constexpr uint32_t kDevErrWaitTimeout = 0x1u;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbarrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

// try_wait with a suspend-time hint: the thread sleeps in hardware until the
// phase completes or `hint_ns` elapses, instead of spinning and stealing
// issue slots from the warps doing real work on the same scheduler.
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar_addr, uint32_t parity,
                                              uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar_addr), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

constexpr uint32_t kWaitHintNs = 200000u;  // 200 us per suspended try_wait

// Waits for the phase of `bar` with the given parity to complete.  Gives up
// after `timeout_ns` of wall time, records the failure in g_frn_device_error
// and in *abort_flag (shared), and returns false.  Also returns false early
// if another role already aborted.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          volatile uint32_t* abort_flag,
                                          uint64_t timeout_ns) {
  const uint32_t a = smem_addr(bar);
  if (mbar_try_wait(a, parity, kWaitHintNs)) return true;
  const uint64_t t0 = global_timer_ns();
  for (;;) {
    if (mbar_try_wait(a, parity, kWaitHintNs)) return true;
    if (*abort_flag) return false;
    if (global_timer_ns() - t0 > timeout_ns) {
      *abort_flag = 1u;
      atomicOr(&g_frn_device_error, kDevErrWaitTimeout);
      return false;
    }
  }
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}

// 2-D tiled TMA load into this CTA's shared memory; completion is signalled
// on `bar` as transaction bytes.  c0 is the innermost (contiguous) coordinate.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* m, uint64_t* bar,
                                            int32_t c0, int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_addr(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_addr(bar)), "r"(c0), "r"(c1)
      : "memory");
}

// 3-D tiled TMA load (coordinates innermost first) into this CTA's shared
// memory; completion is signalled on `bar` as transaction bytes.
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* m, uint64_t* bar,
                                            int32_t c0, int32_t c1, int32_t c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_addr(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_addr(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// Warms L2 with a 2-D tile (no shared memory written, nothing to wait for).
// Safe before griddepcontrol.wait: L2 is the coherence point, so a line
// fetched before the preceding grid writes it is simply updated by that write.
__device__ __forceinline__ void tma_prefetch_2d(const CUtensorMap* m, int32_t c0, int32_t c1) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
                   reinterpret_cast<uint64_t>(m)),
               "r"(c0), "r"(c1)
               : "memory");
}

// 2-D tiled TMA store from shared memory (bulk-group completion).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* m, const void* smem_src,
                                             int32_t c0, int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(m)),
      "r"(smem_addr(smem_src)), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void bulk_wait_group_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// Orders this thread's generic-proxy shared-memory writes before later
// async-proxy (TMA) reads of the same memory.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_addr(smem_result)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D(tmem) (+)= A(smem) * B(smem)^T, both K-major, described by 64-bit smem
// descriptors; idesc is the 32-bit instruction descriptor.
__device__ __forceinline__ void umma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive (once) on `bar` when all previously issued tcgen05 ops of this
// thread have completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_addr(bar))
               : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread t of the warp receives
// lane (warp_quarter*32 + t), columns [col, col+32).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ---------------------------------------------------------------- clusters / CTA pairs
__device__ __forceinline__ uint32_t cluster_cta_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// shared::cluster address of the same shared variable in CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t local_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_addr), "r"(rank));
  return r;
}

// Relaxed remote arrive: no memory ordering beyond the barrier itself.  Used
// where the only thing to order is tcgen05 work, which the caller fences with
// tcgen05.fence::before_thread_sync; avoids waiting for outstanding stores.
__device__ __forceinline__ void mbar_arrive_cluster_relaxed(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar_addr, uint32_t parity,
                                                      uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar_addr), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// mbar_wait for barriers that receive arrivals from the peer CTA.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity,
                                                  volatile uint32_t* abort_flag,
                                                  uint64_t timeout_ns) {
  const uint32_t a = smem_addr(bar);
  if (mbar_try_wait_cluster(a, parity, kWaitHintNs)) return true;
  const uint64_t t0 = global_timer_ns();
  for (;;) {
    if (mbar_try_wait_cluster(a, parity, kWaitHintNs)) return true;
    if (*abort_flag) return false;
    if (global_timer_ns() - t0 > timeout_ns) {
      *abort_flag = 1u;
      atomicOr(&g_frn_device_error, kDevErrWaitTimeout);
      return false;
    }
  }
}

// Full cluster barrier (all threads of all CTAs), not warp-aligned.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

// 4-byte store into a peer CTA's shared memory whose completion is signalled
// as 4 transaction bytes on the peer's mbarrier.  The complete_tx has
// cluster-scope release semantics, so the peer thread that acquires that
// barrier phase also sees this thread's earlier writes -- without this thread
// waiting for them as a releasing remote arrive would.
__device__ __forceinline__ void st_async_complete_tx(uint32_t remote_addr, uint32_t value,
                                                     uint32_t remote_bar) {
  asm volatile(
      "st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(
          remote_addr),
      "r"(value), "r"(remote_bar)
      : "memory");
}

// Cluster rendezvous without release semantics on the arrive.  For points
// where every cross-CTA write of this thread has already been observed by its
// target (or was released by a fence such as fence.mbarrier_init), so only
// the execution barrier is needed; a releasing arrive costs a cluster-scope
// memory fence while the SM still has global stores draining.
__device__ __forceinline__ void cluster_sync_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

// The two halves of a cluster rendezvous, for a thread that has other work
// between announcing it is ready and needing everyone else to be.
// Named CTA barrier `id` (1..15) over `count` threads (a multiple of 32).
__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed;" ::: "memory");
}
__device__ __forceinline__ void cluster_arrive_release() {
  asm volatile("barrier.cluster.arrive.release;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire;" ::: "memory");
}

// 4-byte store into the shared memory of any CTA of the cluster
// (`cluster_addr` from mapa_shared).
__device__ __forceinline__ void st_shared_cluster_f32(uint32_t cluster_addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(cluster_addr), "f"(v) : "memory");
}

// 2-D tiled TMA load for a CTA pair: data lands in this CTA's smem, the
// transaction bytes are signalled on `bar_cluster_addr`, which may be the
// mbarrier of either CTA of the pair.
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* m,
                                                 uint32_t bar_cluster_addr, int32_t c0,
                                                 int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_addr(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(bar_cluster_addr), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_addr(smem_result)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// D(tmem, both CTAs) (+)= A(smem, both CTAs) * B(smem, both CTAs)^T with
// M = 256 across the pair; issued by one thread of the even CTA.
__device__ __forceinline__ void umma_f16_ss_pair(uint32_t d_tmem, uint64_t a_desc,
                                                 uint64_t b_desc, uint32_t idesc,
                                                 uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on the mbarrier at this offset in every CTA of `cta_mask` when
// all prior tcgen05 ops of this thread (pair MMAs included) have completed.
__device__ __forceinline__ void umma_commit_pair_mc(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(smem_addr(bar)),
      "h"(cta_mask)
      : "memory");
}

__device__ __forceinline__ void griddep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// 16-byte store to this CTA's shared memory by shared-window address (keeps
// the access an STS even where the compiler has lost the address space).
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
               "r"(d));
}

__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}

__device__ __forceinline__ float ld_shared_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr));
  return v;
}

__device__ __forceinline__ float4 ld_shared_v4f(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr));
  return v;
}

// 16-byte read-only global load (non-coherent path).
__device__ __forceinline__ uint4 ld_global_nc_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// ---------------------------------------------------------------- descriptors
// Shared-memory matrix descriptor for a K-major operand tile stored the way a
// 128-byte-swizzled TMA load leaves it: rows of 128 bytes (64 16-bit
// elements), groups of 8 rows 1024 bytes apart, tile base 1024-aligned.
// Fields (tcgen05 smem descriptor): start address >> 4 at [0,14), leading
// byte offset >> 4 at [16,30) (unused for swizzled K-major; 1), stride byte
// offset >> 4 at [32,46), descriptor version 1 at [46,48), swizzle mode at
// [61,64) with 2 = 128-byte swizzle.
__device__ __forceinline__ uint64_t make_smem_desc_k_sw128(uint32_t smem_byte_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_byte_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;
  d |= static_cast<uint64_t>(1024u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}

// Instruction descriptor for kind::f16 with fp32 accumulation, both operands
// K-major.  ab_format: 0 = fp16, 1 = bf16.  Fields: c_format [4,6) (1 = f32),
// a_format [7,10), b_format [10,13), a_major bit 15, b_major bit 16,
// N >> 3 at [17,23), M >> 4 at [24,29).
__host__ __device__ constexpr uint32_t make_idesc_f16(uint32_t ab_format, uint32_t m,
                                                      uint32_t n) {
  return (1u << 4) | (ab_format << 7) | (ab_format << 10) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

// Operand format code of the kind::f16 instruction descriptor and the TMA
// element type for each 16-bit input type.
template <typename T>
struct Elem16;
template <>
struct Elem16<__nv_bfloat16> {
  static constexpr uint32_t kUmmaFormat = 1u;
  static constexpr CUtensorMapDataType kTmaType = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
};
template <>
struct Elem16<__half> {
  static constexpr uint32_t kUmmaFormat = 0u;
  static constexpr CUtensorMapDataType kTmaType = CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
};

// ---------------------------------------------------------------- misc
__device__ __forceinline__ uint32_t warp_id_in_cta() {
  return __shfl_sync(0xffffffffu, threadIdx.x / 32u, 0);
}

__device__ __forceinline__ float2 bf162_to_float2(uint32_t v) {
  __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&v);
  return __bfloat1622float2(b);
}

__device__ __forceinline__ float2 half2_to_float2(uint32_t v) {
  __half2 h = *reinterpret_cast<__half2*>(&v);
  return __half22float2(h);
}

template <typename T>
__device__ __forceinline__ float2 pair_to_float2(uint32_t v);
template <>
__device__ __forceinline__ float2 pair_to_float2<__nv_bfloat16>(uint32_t v) {
  return bf162_to_float2(v);
}
template <>
__device__ __forceinline__ float2 pair_to_float2<__half>(uint32_t v) {
  return half2_to_float2(v);
}

template <typename T>
__device__ __forceinline__ uint32_t float2_to_pair(float a, float b);
template <>
__device__ __forceinline__ uint32_t float2_to_pair<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 r = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&r);
}
template <>
__device__ __forceinline__ uint32_t float2_to_pair<__half>(float a, float b) {
  __half2 r = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&r);
}

// Epilogue staging for a TMA tensor store.  Lane r holds row r of a warp's
// 32-row block as fp32 accumulator columns v[0 .. 8*NJ); each value is
// multiplied by `scale` (the row's inv_rms) and, with COLSCALE, by the
// column's factor read from shared memory at `colscale` (8*NJ floats),
// optionally gets the bias columns bv[j] (8 values of T per 16-byte chunk)
// added, is rounded once to T, and is written to the block at `sb` in the
// swizzled layout the store's tensor map names:
//   NJ = 8: rows of 128 B, 128-byte swizzle: chunk j of row r at
//           r*128 + 16*(j ^ (r & 7))           (block 1024-byte aligned)
//   NJ = 4: rows of 64 B, 64-byte swizzle:   chunk j of row r at
//           r*64 + 16*(j ^ ((r >> 1) & 3))     (block 512-byte aligned)
// Both patterns put the 8 lanes of each shared-memory phase on distinct banks.
template <typename T, int NJ, bool BIAS, bool COLSCALE = false>
__device__ __forceinline__ void stage_rows_swizzled(const uint32_t (&v)[64], float scale,
                                                    const uint4 (&bv)[8], uint32_t sb,
                                                    uint32_t lane, uint32_t colscale = 0) {
  static_assert(NJ == 8 || NJ == 4, "64- or 32-column blocks");
#pragma unroll
  for (int j = 0; j < NJ; ++j) {
    float f[8];
    if (COLSCALE) {
      const float4 c0 = ld_shared_v4f(colscale + j * 32), c1 = ld_shared_v4f(colscale + j * 32 + 16);
      const float cs[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
#pragma unroll
      for (int e = 0; e < 8; ++e) f[e] = __uint_as_float(v[j * 8 + e]) * cs[e] * scale;
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) f[e] = __uint_as_float(v[j * 8 + e]) * scale;
    }
    if (BIAS) {
      const float2 b0 = pair_to_float2<T>(bv[j].x), b1 = pair_to_float2<T>(bv[j].y);
      const float2 b2 = pair_to_float2<T>(bv[j].z), b3 = pair_to_float2<T>(bv[j].w);
      f[0] += b0.x; f[1] += b0.y; f[2] += b1.x; f[3] += b1.y;
      f[4] += b2.x; f[5] += b2.y; f[6] += b3.x; f[7] += b3.y;
    }
    const uint32_t off = NJ == 8 ? lane * 128u + ((static_cast<uint32_t>(j) ^ (lane & 7u)) << 4)
                                 : lane * 64u + ((static_cast<uint32_t>(j) ^ ((lane >> 1) & 3u)) << 4);
    st_shared_v4(sb + off, float2_to_pair<T>(f[0], f[1]), float2_to_pair<T>(f[2], f[3]),
                 float2_to_pair<T>(f[4], f[5]), float2_to_pair<T>(f[6], f[7]));
  }
}

// SwiGLU variant: 32 columns of the gate (gv) and up (uv) accumulators of the
// lane's row -> silu(g * scale + b_g) * (u * scale + b_u), rounded once to T,
// written as 16-byte chunks jbase .. jbase+3 of the row in the same swizzled
// layouts as stage_rows_swizzled (NJ = 8: 128-byte rows, NJ = 4: 64-byte).
// silu(a) = a / (1 + e^-a), with the fast exponential and division.
template <typename T, int NJ, bool BIAS>
__device__ __forceinline__ void stage_swiglu_rows(const uint32_t (&gv)[32],
                                                  const uint32_t (&uv)[32], float scale,
                                                  const uint4 (&bg)[4], const uint4 (&bu)[4],
                                                  uint32_t sb, uint32_t lane, int jbase) {
  static_assert(NJ == 8 || NJ == 4, "64- or 32-column blocks");
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float g[8], u[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      g[e] = __uint_as_float(gv[j * 8 + e]) * scale;
      u[e] = __uint_as_float(uv[j * 8 + e]) * scale;
    }
    if (BIAS) {
      const uint32_t bgw[4] = {bg[j].x, bg[j].y, bg[j].z, bg[j].w};
      const uint32_t buw[4] = {bu[j].x, bu[j].y, bu[j].z, bu[j].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 a = pair_to_float2<T>(bgw[e]), b = pair_to_float2<T>(buw[e]);
        g[2 * e] += a.x; g[2 * e + 1] += a.y;
        u[2 * e] += b.x; u[2 * e + 1] += b.y;
      }
    }
    float f[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) f[e] = __fdividef(g[e], 1.0f + __expf(-g[e])) * u[e];
    const uint32_t jj = static_cast<uint32_t>(jbase + j);
    const uint32_t off = NJ == 8 ? lane * 128u + ((jj ^ (lane & 7u)) << 4)
                                 : lane * 64u + ((jj ^ ((lane >> 1) & 3u)) << 4);
    st_shared_v4(sb + off, float2_to_pair<T>(f[0], f[1]), float2_to_pair<T>(f[2], f[3]),
                 float2_to_pair<T>(f[4], f[5]), float2_to_pair<T>(f[6], f[7]));
  }
}

}  // namespace frn
