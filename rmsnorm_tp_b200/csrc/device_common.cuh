// Device helpers shared by the forward kernels (kernels.cu) and the backward
// kernels (backward.cu): 16-byte element packing, warp sums, and one lane's
// share of the cross-GPU exchange (push a partial into a peer's mailbox slot,
// poll the local slot with a bounded wait), plus the generation bookkeeping.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "internal.h"
#include "ptx.cuh"
#include "rtp_common.h"

namespace rtp {

// ---------------------------------------------------------------------------
// Element packing: 16 bytes = 4 fp32 or 8 bf16/fp16.
// ---------------------------------------------------------------------------
template <typename T>
struct Pack;

template <>
struct Pack<float> {
  static constexpr int kE = 4;
  __device__ __forceinline__ static void unpack(const uint4& v, float (&f)[4]) {
    f[0] = __uint_as_float(v.x);
    f[1] = __uint_as_float(v.y);
    f[2] = __uint_as_float(v.z);
    f[3] = __uint_as_float(v.w);
  }
  __device__ __forceinline__ static uint4 pack(const float (&f)[4]) {
    return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]),
                      __float_as_uint(f[3]));
  }
  __device__ __forceinline__ static float to_f(float v) { return v; }
  __device__ __forceinline__ static float from_f(float v) { return v; }
};

__device__ __forceinline__ void bf16x2_unpack(uint32_t u, float& lo, float& hi) {
  lo = __uint_as_float(u << 16);
  hi = __uint_as_float(u & 0xFFFF0000u);
}
__device__ __forceinline__ uint32_t bf16x2_pack(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

template <>
struct Pack<__nv_bfloat16> {
  static constexpr int kE = 8;
  __device__ __forceinline__ static void unpack(const uint4& v, float (&f)[8]) {
    bf16x2_unpack(v.x, f[0], f[1]);
    bf16x2_unpack(v.y, f[2], f[3]);
    bf16x2_unpack(v.z, f[4], f[5]);
    bf16x2_unpack(v.w, f[6], f[7]);
  }
  __device__ __forceinline__ static uint4 pack(const float (&f)[8]) {
    return make_uint4(bf16x2_pack(f[0], f[1]), bf16x2_pack(f[2], f[3]), bf16x2_pack(f[4], f[5]),
                      bf16x2_pack(f[6], f[7]));
  }
  __device__ __forceinline__ static float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  __device__ __forceinline__ static __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};

__device__ __forceinline__ void f16x2_unpack(uint32_t u, float& lo, float& hi) {
  __half2 h = *reinterpret_cast<__half2*>(&u);
  float2 f = __half22float2(h);
  lo = f.x;
  hi = f.y;
}
__device__ __forceinline__ uint32_t f16x2_pack(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

template <>
struct Pack<__half> {
  static constexpr int kE = 8;
  __device__ __forceinline__ static void unpack(const uint4& v, float (&f)[8]) {
    f16x2_unpack(v.x, f[0], f[1]);
    f16x2_unpack(v.y, f[2], f[3]);
    f16x2_unpack(v.z, f[4], f[5]);
    f16x2_unpack(v.w, f[6], f[7]);
  }
  __device__ __forceinline__ static uint4 pack(const float (&f)[8]) {
    return make_uint4(f16x2_pack(f[0], f[1]), f16x2_pack(f[2], f[3]), f16x2_pack(f[4], f[5]),
                      f16x2_pack(f[6], f[7]));
  }
  __device__ __forceinline__ static float to_f(__half v) { return __half2float(v); }
  __device__ __forceinline__ static __half from_f(float v) { return __float2half_rn(v); }
};

// Butterfly sum: every lane ends with the bit-identical total (IEEE addition is
// commutative, and each step adds the same two operands on both partner lanes).
__device__ __forceinline__ float warp_allreduce_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

template <typename T>
__device__ __forceinline__ float sumsq16(const uint4& v) {
  float f[Pack<T>::kE];
  Pack<T>::unpack(v, f);
  float a = 0.f, b = 0.f;
#pragma unroll
  for (int e = 0; e < Pack<T>::kE; e += 2) {
    a = fmaf(f[e], f[e], a);
    b = fmaf(f[e + 1], f[e + 1], b);
  }
  return a + b;
}

template <typename T>
__device__ __forceinline__ uint4 normalize16(const uint4& xv, const uint4& wv, float inv) {
  float xf[Pack<T>::kE], wf[Pack<T>::kE];
  Pack<T>::unpack(xv, xf);
  Pack<T>::unpack(wv, wf);
#pragma unroll
  for (int e = 0; e < Pack<T>::kE; ++e) xf[e] = (xf[e] * inv) * wf[e];
  return Pack<T>::pack(xf);
}

// Fused residual add: z = x + r in fp32, rounded once to T.
template <typename T>
__device__ __forceinline__ uint4 add16(const uint4& xv, const uint4& rv) {
  float xf[Pack<T>::kE], rf[Pack<T>::kE];
  Pack<T>::unpack(xv, xf);
  Pack<T>::unpack(rv, rf);
#pragma unroll
  for (int e = 0; e < Pack<T>::kE; ++e) xf[e] += rf[e];
  return Pack<T>::pack(xf);
}

__device__ __forceinline__ float quiet_nan() { return __uint_as_float(0x7FC00000u); }

// ---------------------------------------------------------------------------
// Cross-GPU exchange, one lane's share, in two steps.
//
// push_slot: store this rank's partial of `row` into rank q's mailbox slot
// [buf][rank][row] (one relaxed system-scope 64-bit store over NVLink).
// poll_slot: wait, bounded by the global timer, until slot [buf][q][row] of the
// local mailbox carries `tag`, and return rank q's partial. Lanes with
// q == rank or !active return `mine`. A timeout is recorded in the rank's
// DeviceState (first failure wins) and mirrored to the host-mapped flag; it
// also raises `abort`, which makes every other wait of this launch give up.
// ---------------------------------------------------------------------------
struct WaitStats {          // optional per-lane counters (KArgs::prof)
  unsigned long long ns = 0;
  unsigned int slow = 0;    // waits that found the slot not yet written
  unsigned int fast = 0;    // waits satisfied by the first poll
};

// Stores {mine, tag} into a slot: one 64-bit system-scope store (packed encoding,
// the default), or the value and then the tag with a release store (the
// reference's flag scheme, KArgs::push_mode == kPushRelease).
__device__ __forceinline__ void store_slot(int push_mode, unsigned long long* dst, float mine,
                                           uint32_t tag) {
  if (push_mode == kPushRelease) {
    unsigned int* w = reinterpret_cast<unsigned int*>(dst);   // [0] value, [1] tag
    ptx::st_relaxed_sys_u32(w, f32_bits(mine));
    ptx::st_release_sys_u32(w + 1, tag);
  } else {
    ptx::st_relaxed_sys_u64(dst, pack_slot(mine, tag));
  }
}

// One look at a local slot: true if it carries `tag`; *word gets {tag seen, value}.
__device__ __forceinline__ bool probe_slot(int push_mode, const unsigned long long* src,
                                           uint32_t tag, unsigned long long* word) {
  if (push_mode == kPushRelease) {
    const unsigned int* w = reinterpret_cast<const unsigned int*>(src);
    const unsigned int t = ptx::ld_acquire_sys_u32(w + 1);
    if (t != tag) {
      *word = (unsigned long long)t << 32;
      return false;
    }
    *word = ((unsigned long long)t << 32) | ptx::ld_relaxed_sys_u32(w);
    return true;
  }
  *word = ptx::ld_relaxed_sys_u64(src);
  return slot_tag(*word) == tag;
}

__device__ __forceinline__ void push_slot(const KArgs& a, int rank, uint32_t buf, uint32_t tag,
                                          int64_t row, int q, bool active, float mine) {
  if (active && q != rank) {
    unsigned long long* dst = a.mbox[q] + slot_index(buf, rank, a.tp, a.nmax, row);
    store_slot(a.push_mode, dst, mine, tag);
  }
}

// Bounded wait until the local slot `src` carries `tag`: kStatusOk, or
// kStatusTimeout after timeout_ns, or kStatusAborted once *abort_flag is set
// (another wait of this GPU gave up). *word gets the last word seen.
__device__ __forceinline__ uint32_t wait_slot(int push_mode, const unsigned long long* src,
                                              uint32_t tag, unsigned long long timeout_ns,
                                              const unsigned int* abort_flag,
                                              unsigned long long* word, WaitStats& ws) {
  if (probe_slot(push_mode, src, tag, word)) {
    ws.fast += 1;
    return kStatusOk;
  }
  uint32_t fail = kStatusOk;
  const unsigned long long t0 = ptx::globaltimer();
  // the abort flag and the timer are looked at every 8 probes: each is a
  // dependent round trip that would otherwise delay seeing the slot arrive
  for (unsigned n = 1;; ++n) {
    if (probe_slot(push_mode, src, tag, word)) break;
    if ((n & 7u) != 0u) continue;
    if (abort_flag != nullptr && ptx::ld_relaxed_gpu_u32(abort_flag) != 0u) {
      fail = kStatusAborted;
      break;
    }
    if (ptx::globaltimer() - t0 > timeout_ns) {
      fail = kStatusTimeout;
      break;
    }
  }
  ws.slow += 1;
  ws.ns += ptx::globaltimer() - t0;
  return fail;
}

__device__ __forceinline__ float poll_slot(const KArgs& a, int rank, const RankPtrs& rp,
                                           uint32_t buf, uint32_t tag, unsigned long long call,
                                           int64_t row, int q, bool active, float mine,
                                           bool& failed, WaitStats& ws) {
  failed = false;
  if (!active || q == rank) return mine;
  const unsigned long long* src = a.mbox[rank] + slot_index(buf, q, a.tp, a.nmax, row);
  unsigned long long w = 0ull;
  const uint32_t fail = wait_slot(a.push_mode, src, tag, a.timeout_ns, &rp.state->abort, &w, ws);
  if (fail == kStatusTimeout) {
    DeviceState* st = rp.state;
    if (atomicCAS(&st->err_code, 0u, (unsigned)kStatusTimeout) == 0u) {
      st->err_src = (unsigned)q;
      st->err_row = (long long)row;
      st->err_expected = tag;
      st->err_seen = slot_tag(w);
      st->err_call = call;
      if (rp.host_flag != nullptr) {
        *reinterpret_cast<volatile unsigned int*>(rp.host_flag) = (unsigned)kStatusTimeout;
        __threadfence_system();
      }
    }
    atomicExch(&st->abort, 1u);
  }
  failed = (fail != kStatusOk);
  return slot_value(w);
}

__device__ __forceinline__ float push_poll(const KArgs& a, int rank, const RankPtrs& rp,
                                           uint32_t buf, uint32_t tag, unsigned long long call,
                                           int64_t row, int q, bool active, float mine,
                                           bool& failed, WaitStats& ws) {
  push_slot(a, rank, buf, tag, row, q, active, mine);
  return poll_slot(a, rank, rp, buf, tag, call, row, q, active, mine, failed, ws);
}

// Wait (bounded) for an mbarrier phase that a bulk copy completes; false when
// the copy has not landed within limit_ns.
constexpr unsigned long long kLoadTimeoutNs = 2000000000ull;   // a bulk copy that never lands

__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity,
                                                  unsigned long long limit_ns) {
  if (ptx::mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = ptx::globaltimer();
  for (;;) {
    if (ptx::mbar_try_wait(bar, parity)) return true;
    if (ptx::globaltimer() - t0 > limit_ns) return false;
  }
}

// Adds the lanes' wait counters and the CTA's timings to KArgs::prof (global
// timer, ns; every CTA of a launch calls this exactly once, at its end, with
// every thread). The CTA's end is stamped once all its threads arrive and
// before any counter is written; the lanes' counters are summed per CTA first
// (warp shuffles, then shared memory), so a CTA makes one global atomic per
// counter and the counters disturb the timings they record as little as possible:
// [0] wait ns summed over lanes, [1] slow waits, [2] fast waits,
// [3] earliest CTA start, [4] latest CTA end,
// [5] sum over CTAs of (t_mid - start), [6] sum of (end - t_mid), [7] CTAs
//     that passed a t_mid (the resident kernel: t_mid = its partials pushed),
// [8] sum over CTAs of (end - start), [9] CTAs,
// [10] sum over launches of (last CTA end - first CTA start), [11] launches,
// [12] sum over launches after the first of (first CTA start - the previous
//      launch's end), [13] launches counted in [12],
// [14]..[16] scratch: this launch's first start (initialise to UINT64_MAX),
//      the previous launch's end, the CTAs of this launch seen so far,
// [17] sum over CTAs of launches after the first of (CTA start - the previous
//      launch's end), [18] CTAs counted in [17], [19] unused.
__device__ __forceinline__ void flush_stats(const KArgs& a, const WaitStats& ws,
                                            unsigned long long t_start,
                                            unsigned long long t_mid = 0ull) {
  if (a.prof == nullptr) return;
  __shared__ unsigned long long s_wait[3];
  if (threadIdx.x == 0) s_wait[0] = s_wait[1] = s_wait[2] = 0ull;
  unsigned long long ns = ws.ns, slow = ws.slow, fast = ws.fast;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    ns += __shfl_xor_sync(0xFFFFFFFFu, ns, o);
    slow += __shfl_xor_sync(0xFFFFFFFFu, slow, o);
    fast += __shfl_xor_sync(0xFFFFFFFFu, fast, o);
  }
  __syncthreads();   // every thread of the CTA is done
  const unsigned long long t_end = ptx::globaltimer();
  if ((threadIdx.x & 31) == 0 && (slow | fast)) {
    atomicAdd(&s_wait[0], ns);
    atomicAdd(&s_wait[1], slow);
    atomicAdd(&s_wait[2], fast);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long* P = a.prof;
    if (s_wait[1]) {
      atomicAdd(P + 0, s_wait[0]);
      atomicAdd(P + 1, s_wait[1]);
    }
    if (s_wait[2]) atomicAdd(P + 2, s_wait[2]);
    atomicMin(P + 3, t_start);
    atomicMax(P + 4, t_end);
    if (t_mid) {
      atomicAdd(P + 5, t_mid - t_start);
      atomicAdd(P + 6, t_end - t_mid);
      atomicAdd(P + 7, 1ull);
    }
    atomicAdd(P + 8, t_end - t_start);
    atomicAdd(P + 9, 1ull);
    // the previous launch's end: stable until this launch's last CTA, which
    // arrives after this one, overwrites it
    const unsigned long long prev = atomicAdd(P + 15, 0ull);
    if (prev != 0ull) {
      atomicAdd(P + 17, t_start > prev ? t_start - prev : 0ull);
      atomicAdd(P + 18, 1ull);
    }
    atomicMin(P + 14, t_start);
    __threadfence();
    const unsigned long long seen = atomicAdd(P + 16, 1ull);
    if (seen == (unsigned long long)gridDim.x * gridDim.y - 1ull) {   // the launch's last CTA
      __threadfence();
      const unsigned long long first = atomicAdd(P + 14, 0ull);
      const unsigned long long prev_end = atomicAdd(P + 15, 0ull);
      atomicAdd(P + 10, t_end - first);
      atomicAdd(P + 11, 1ull);
      if (prev_end != 0ull) {
        atomicAdd(P + 12, first > prev_end ? first - prev_end : 0ull);
        atomicAdd(P + 13, 1ull);
      }
      atomicExch(P + 15, t_end);
      atomicExch(P + 14, ~0ull);
      atomicExch(P + 16, 0ull);
    }
  }
}

// Advances the rank's generation counter by `step` (one per exchange the launch
// made: forward and linear 1, backward 2; see DeviceState) once every thread of
// the CTA has read it. One generation: this CTA's share, a reduction whose
// result is unused (red.global.add) -- no CTA waits for it. Two: the last CTA
// of the launch (a returning atomic on `done`) stores the advanced value. The
// next launch reads the counter only once this grid has completed (stream
// order, or its griddepcontrol.wait), when every write of the grid is visible.
// No fence: one would hold each CTA's exit until its outstanding stores, the
// pushes to peers included, were acknowledged.
__device__ __forceinline__ void finish_launch(DeviceState* st, unsigned long long call,
                                              unsigned long long step = 1ull) {
  __syncthreads();
  if (threadIdx.x != 0) return;
  if (step == 1ull) {
    atomicAdd(&st->call, (unsigned long long)gen_share(blockIdx.x, gridDim.x));
  } else if (atomicAdd(&st->done, 1u) == gridDim.x - 1u) {
    st->done = 0u;
    st->call = (call + step) << kGenShift;
  }
}

// The generation of the running launch (read before the CTA adds its share).
__device__ __forceinline__ unsigned long long read_generation(const DeviceState* st) {
  return gen_of(*reinterpret_cast<const volatile unsigned long long*>(&st->call));
}

}  // namespace rtp
