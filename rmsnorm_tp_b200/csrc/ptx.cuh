// Inline-PTX memory primitives for sm_100a.
//
// The reference uses st.release.sys for a separate generation flag and
// ld.volatile + ld.acquire.sys to poll it (csrc/rmsnorm_tp.cu:11-29). Here the
// partial sum and its tag share one naturally aligned 64-bit word, so relaxed
// system-scope accesses are enough: a load that observes the tag observes the
// value written by the same single-copy-atomic store.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace rtp {
namespace ptx {

// Streaming 128-bit load of data read once (x rows, the residual): no L1
// allocation. A coherent load, not the read-only (.nc) path: the kernel may
// write the same memory (out == x in place, the residual rewritten with
// x + residual), which the read-only path does not allow within one kernel.
__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
  uint4 v;
  asm("ld.global.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
      : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
      : "l"(p));
  return v;
}

// 128-bit load of data every warp of the SM re-reads and no kernel writes (the
// weight): read-only path, L1-cached.
__device__ __forceinline__ uint4 ld_cached_v4(const void* p) {
  uint4 v;
  asm("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];"
      : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
      : "l"(p));
  return v;
}

// Brings the line holding p into L1 (no register, nothing waits for it).
__device__ __forceinline__ void prefetch_l1(const void* p) {
  asm volatile("prefetch.global.L1 [%0];" ::"l"(p));
}

__device__ __forceinline__ void st_v4(void* p, const uint4& v) {
  asm volatile("st.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

// Mailbox push into a peer's (or this GPU's) memory.
__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Mailbox poll of this GPU's memory (peers write it over NVLink).
__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// The reference's push encoding (csrc/rmsnorm_tp.cu:102-115, :121-138): the value
// with a plain system-scope store, then a separate flag word with a release
// store; the reader acquires the flag, then reads the value. Kept for the
// measured comparison with the packed 64-bit word (push encoding 1).
__device__ __forceinline__ void st_relaxed_sys_u32(unsigned int* p, unsigned int v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_release_sys_u32(unsigned int* p, unsigned int v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned int ld_acquire_sys_u32(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned int ld_relaxed_sys_u32(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ unsigned int ld_relaxed_gpu_u32(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_relaxed_gpu_u32(unsigned int* p, unsigned int v) {
  asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Nanosecond wall clock of the GPU; bounds every wait.
__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---- shared-memory barriers and bulk (TMA) copies --------------------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

// Makes mbarrier initialisation visible to the async (bulk copy) proxy.
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Orders this thread's earlier generic-proxy shared-memory accesses before
// later async-proxy (bulk copy) accesses of the same memory.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0u;
}

// 1-D bulk copy global -> this CTA's shared memory, completion counted in bytes
// on `bar`. Source is this GPU's own memory; dst, src and bytes are multiples of 16.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes,
                                          uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

// Programmatic dependent launch. grid_dep_wait: block until every grid this
// launch depends on programmatically has completed and its memory operations
// are visible (returns at once for a launch without such a dependency); no
// global memory is touched before it. grid_dep_launch_dependents: allow the
// next launch in the stream to start being scheduled (its CTAs fill SMs as
// this grid's CTAs exit, and wait in their own grid_dep_wait).
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Returns p unchanged, through a volatile asm: loads through the result are
// data-dependent on this point, so the (non-volatile) load asm above cannot be
// scheduled before a preceding grid_dep_wait.
template <typename P>
__device__ __forceinline__ P* launder(P* p) {
  asm volatile("" : "+l"(p));
  return p;
}

// Barrier over the `nthreads` threads of one team (named barrier `id`, 1..15).
__device__ __forceinline__ void team_bar(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

}  // namespace ptx
}  // namespace rtp
