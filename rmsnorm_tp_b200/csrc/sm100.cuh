// Blackwell (sm_100a) tensor-core primitives for the fused row-parallel
// linear -> reduce-scatter -> TP RMSNorm kernel (linear.cu): tensor memory
// (TMEM) allocation, tcgen05.mma issue and completion, TMEM -> register loads,
// and 2-D TMA tile loads. Inline PTX; descriptor bit layouts follow the PTX ISA
// (tcgen05 shared-memory and instruction descriptors).
//
// Every TMA load here reads this GPU's own memory and has no cluster
// multicast qualifier.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace rtp {
namespace sm100 {

// ---- tensor memory ---------------------------------------------------------
// One full warp allocates `ncols` (a power of two >= 32) TMEM columns and
// writes the base address into shared memory at `dst` (a shared address).
__device__ __forceinline__ void tmem_alloc(uint32_t dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst),
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

// Ordering of tcgen05 operations across a thread synchronisation (mbarrier or
// bar.sync): `before` in the thread that signals, `after` in the one that waits.
__device__ __forceinline__ void fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (bf16/fp16 inputs, fp32
// accumulate), issued by one thread. accumulate = 0 overwrites D.
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on the mbarrier (shared address) when every tcgen05.mma this
// thread issued before has completed.
__device__ __forceinline__ void mma_commit(uint32_t mbar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   mbar)
               : "memory");
}

// 32 TMEM lanes x 32 columns of 32 bits: thread i of the warp gets lane
// (base lane + i), columns [col, col + 32). The warp may only address the
// 32-lane quarter (warp id % 4) of TMEM.
__device__ __forceinline__ void tmem_ld_32x32(uint32_t taddr, uint32_t (&r)[32]) {
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
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ---- TMA ---------------------------------------------------------------------
// 2-D tiled load of the box at (c0 = innermost coordinate, c1) of the tensor
// map into shared memory, completion counted in bytes on `mbar`. No multicast.
// c0 * element size must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void* tmap, int32_t c0,
                                            int32_t c1, uint32_t mbar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(tmap), "r"(mbar), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void tma_prefetch_desc(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// ---- descriptors -------------------------------------------------------------
// Shared-memory matrix descriptor of a K-major tile whose rows are 128 bytes
// (64 bf16/fp16) stored with the 128-byte swizzle, 8-row atoms of 1024 bytes:
// start address >> 4 in bits [0, 14), leading byte offset >> 4 (unused by the
// swizzled K-major layout, 16 bytes) in [16, 30), stride byte offset >> 4
// (1024 bytes between 8-row atoms) in [32, 46), descriptor version 1 in
// [46, 48), base offset 0, layout type 2 (128-byte swizzle) in [61, 64).
// The tile's base must be 1024-byte aligned; stepping along K inside the
// 128-byte row moves the start address by the step's bytes.
__device__ __forceinline__ uint64_t desc_k_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
  d |= (uint64_t)(16u >> 4) << 16;
  d |= (uint64_t)(1024u >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor of kind::f16 with fp32 accumulation, A and B of the
// same 16-bit type (is_bf16: bf16, else fp16), both K-major, shape M x N:
// D format (F32 = 1) in bits [4, 6), A format in [7, 10), B format in [10, 13),
// N >> 3 in [17, 23), M >> 4 in [24, 29).
__host__ __device__ constexpr uint32_t idesc_f16(bool is_bf16, int m, int n) {
  return (1u << 4) | ((is_bf16 ? 1u : 0u) << 7) | ((is_bf16 ? 1u : 0u) << 10) |
         ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

}  // namespace sm100
}  // namespace rtp
