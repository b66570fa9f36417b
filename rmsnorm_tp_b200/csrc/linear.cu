// Fused row-parallel linear -> reduce-scatter -> (residual add) -> TP RMSNorm
// for B200 (sm_100a), one persistent kernel per call.
//
// In a Megatron-style tensor-parallel block the row-parallel linear (attention
// output projection, MLP down projection) leaves every rank with a partial
// product P_r = A_r W_r^T of the full hidden width, which an all-reduce (or a
// reduce-scatter when the norm is itself tensor parallel) sums before the
// norm. Here rank r:
//   phase 1 -- computes P_r tile by tile on the tensor cores (128 x 128 tiles,
//              tcgen05.mma with fp32 accumulators in tensor memory, operands
//              staged by TMA from this GPU's own memory) and stores each tile,
//              rounded to the dtype, straight into the receive buffer of the
//              rank that owns its columns (peer memory over NVLink, or local),
//              then raises that tile's flag there: the transfer of tile t
//              overlaps the math of the next tiles;
//   phase 2 -- once every rank's tiles of a 128-row block have landed, sums the
//              tp partials of each of its rows in rank order (fp32), rounds
//              to the dtype (x), adds the residual (z = x + residual, written
//              back), and normalises its hl = hidden / tp columns with the
//              one-scalar-per-row exchange of the forward kernels
//              (y = (z * rsqrt(S / hidden + eps)) * gamma, S summed in rank
//              order).
// The reference leaves this step to torch: the partial output goes through
// NCCL, then its AllReduce TP RMSNorm (bench_rmsnorm_tp.py:16-22) normalises.
//
// Roles in phase 1 (192 threads): warp 0 lane 0 issues TMA loads into a ring of
// 4 stages (A and W tiles of 128 x 64); warp 1 allocates tensor memory (two
// 128-column fp32 accumulators) and its lane 0 issues the MMAs; warps 2-5
// (one per 32-lane quarter of tensor memory) read an accumulator, convert it,
// stage it in shared memory and store it to the owner with 16-byte stores
// (512 contiguous bytes per warp instruction). All CTAs are resident (one per
// SM) and phase 1 waits on nothing outside the CTA, so every phase-2 wait on
// another rank's flags or partial sums ends.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstddef>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "device_common.cuh"
#include "internal.h"
#include "ptx.cuh"
#include "rtp_common.h"
#include "sm100.cuh"

namespace rtp {

namespace {
constexpr int kLinThreads = 192;
constexpr uint32_t kLinPitch = 128 * 2 + 16;                        // staging row: 256 + 16 bytes
constexpr uint32_t kLinStagingBytes = kLinTileM * kLinPitch;        // 128 columns at a time
constexpr unsigned long long kLinWaitNs = 2000000000ull;           // an internal wait that never ends

// Tile shapes: 128 rows x kBN columns (64, 128 or 256) per tile, 64-element K
// steps. 256-column tiles load 48 KB per K step for 4.2 MFLOP (128-column: 32 KB
// for 2.1 MFLOP), so they need less L2 bandwidth per FLOP; they take the whole
// tensor memory (two 256-column fp32 accumulators) and 3 ring stages. 64-column
// tiles serve calls of few row blocks, where wider tiles would leave most SMs
// idle while the weights stream from HBM (6 stages of 24 KB in flight).
template <int kBN>
struct LinCfg {
  static_assert(kBN == 64 || kBN == 128 || kBN == 256, "tile width");
  static constexpr int kStages = kBN == 256 ? 3 : kBN == 128 ? 4 : 6;
  static constexpr uint32_t kABytes = kLinTileM * kLinTileK * 2;    // 16 KB
  static constexpr uint32_t kBBytes = kBN * kLinTileK * 2;          // 16 or 32 KB
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  static constexpr uint32_t kSmem = 1024 + kStages * kStageBytes + kLinStagingBytes;
  static constexpr uint32_t kTmemCols = 2 * kBN;
};

__device__ __forceinline__ bool wait_bounded(uint32_t bar, uint32_t parity) {
  if (ptx::mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = ptx::globaltimer();
  for (;;) {
    if (ptx::mbar_try_wait(bar, parity)) return true;
    if (ptx::globaltimer() - t0 > kLinWaitNs) return false;
  }
}

__device__ __forceinline__ void record_failure(DeviceState* st, unsigned int* host_flag,
                                               unsigned code, unsigned long long call) {
  if (st == nullptr) return;
  if (atomicCAS(&st->err_code, 0u, code) == 0u) {
    st->err_call = call;
    if (host_flag != nullptr) {
      *reinterpret_cast<volatile unsigned int*>(host_flag) = code;
      __threadfence_system();
    }
  }
  atomicExch(&st->abort, 1u);
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  return bf16x2_pack(lo, hi);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
  return f16x2_pack(lo, hi);
}
}  // namespace

template <typename T, int kBN>
__global__ void __launch_bounds__(kLinThreads, 1)
    tp_linear_rmsnorm_kernel(const __grid_constant__ LArgs a) {
  using Cfg = LinCfg<kBN>;
  constexpr int kLinStages = Cfg::kStages;
  constexpr uint32_t kLinStageBytes = Cfg::kStageBytes;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  __shared__ __align__(8) unsigned long long s_full[kLinStages];
  __shared__ __align__(8) unsigned long long s_empty[kLinStages];
  __shared__ __align__(8) unsigned long long s_accf[2];
  __shared__ __align__(8) unsigned long long s_acce[2];
  __shared__ __align__(8) unsigned long long s_drain;
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort;
  __shared__ unsigned long long s_call;

  ptx::grid_dep_wait();
  ptx::grid_dep_launch_dependents();
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int ri = a.emulated ? (int)blockIdx.y : 0;
  const int rank = a.emulated ? (int)blockIdx.y : a.rank;
  const LinRank& rk = a.rk[ri];
  const int tp = a.tp;
  const bool exchange = tp > 1;
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023u) & ~(uintptr_t)1023u);
  const uint32_t sbase = ptx::smem_addr(smem);
  unsigned char* staging = smem + kLinStages * kLinStageBytes;
  const uint32_t bar_full = ptx::smem_addr(&s_full[0]);
  const uint32_t bar_empty = ptx::smem_addr(&s_empty[0]);
  const uint32_t bar_accf = ptx::smem_addr(&s_accf[0]);
  const uint32_t bar_acce = ptx::smem_addr(&s_acce[0]);
  const uint32_t bar_drain = ptx::smem_addr(&s_drain);

  const int64_t mt = (a.rows + kLinTileM - 1) / kLinTileM;
  const int64_t nt = a.hidden / kBN;
  const int64_t nbl = a.nblocks;                       // column tiles per owner
  const int64_t tiles = mt * nt;
  const int kbs = (int)(a.k / kLinTileK);
  const int64_t hl = a.hl;
  // tile t -> (m block, n block): grouped m blocks, owners dealt in turn
  auto tile_mn = [&](int64_t t, int64_t& mb, int64_t& nb) { linear_tile(t, mt, nt, tp, nbl, &mb, &nb); };

  if (threadIdx.x == 0) {
    for (int s = 0; s < kLinStages; ++s) {
      ptx::mbar_init(bar_full + 8u * s, 1u);
      ptx::mbar_init(bar_empty + 8u * s, 1u);
    }
    for (int c = 0; c < 2; ++c) {
      ptx::mbar_init(bar_accf + 8u * c, 1u);
      ptx::mbar_init(bar_acce + 8u * c, 4u);           // one arrive per epilogue warp
    }
    ptx::mbar_init(bar_drain, 1u);
    ptx::fence_mbar_init();
    s_abort = 0;
    s_call = exchange ? read_generation(rk.state) : 0ull;
  }
  if (warp == 1) {
    sm100::tmem_alloc(ptx::smem_addr(&s_tmem), Cfg::kTmemCols);
    sm100::tmem_relinquish();
    sm100::fence_before_sync();
  }
  __syncthreads();
  sm100::fence_after_sync();
  const uint32_t tmem = s_tmem;
  const unsigned long long call = s_call;
  const uint32_t buf = buffer_of(call), tag = tag_of(call);

  // ------------------------------------------------------------------ phase 1
  if (warp == 0 && lane == 0) {
    // TMA producer
    const void* tma = a.tmaps[2 * ri];
    const void* tmb = a.tmaps[2 * ri + 1];
    sm100::tma_prefetch_desc(tma);
    sm100::tma_prefetch_desc(tmb);
    int64_t it = 0;
    int issued[kLinStages] = {};
    bool ok = true;
    for (int64_t t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
      int64_t mb, nb;
      tile_mn(t, mb, nb);
      for (int kb = 0; kb < kbs; ++kb, ++it) {
        const int s = (int)(it % kLinStages);
        const uint32_t ph = (uint32_t)((it / kLinStages) & 1);
        if (!wait_bounded(bar_empty + 8u * s, ph ^ 1u) || s_abort) {
          ok = false;
          break;
        }
        const uint32_t sa = sbase + (uint32_t)s * kLinStageBytes;
        ptx::mbar_arrive_expect_tx(bar_full + 8u * s, kLinStageBytes);
        sm100::tma_load_2d(sa, tma, kb * kLinTileK, (int32_t)(mb * kLinTileM), bar_full + 8u * s);
        sm100::tma_load_2d(sa + Cfg::kABytes, tmb, kb * kLinTileK, (int32_t)(nb * kBN),
                           bar_full + 8u * s);
        issued[s] += 1;
      }
    }
    if (!ok) {
      s_abort = 1;
      record_failure(rk.state, rk.host_flag, kStatusLoadTimeout, call);
      // the copies already issued land before shared memory is released
      for (int s = 0; s < kLinStages; ++s)
        if (issued[s] > 0) wait_bounded(bar_full + 8u * s, (uint32_t)((issued[s] - 1) & 1));
    }
  } else if (warp == 1 && lane == 0) {
    // MMA issuer
    const uint32_t idesc = sm100::idesc_f16(sizeof(T) == 2 && std::is_same<T, __nv_bfloat16>::value,
                                            kLinTileM, kBN);
    int64_t it = 0, tc = 0;
    bool ok = true;
    for (int64_t t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++tc) {
      const int acc = (int)(tc & 1);
      const uint32_t aph = (uint32_t)((tc >> 1) & 1);
      if (!wait_bounded(bar_acce + 8u * acc, aph ^ 1u) || s_abort) {
        ok = false;
        break;
      }
      sm100::fence_after_sync();
      const uint32_t d = tmem + (uint32_t)(acc * kBN);
      for (int kb = 0; kb < kbs; ++kb, ++it) {
        const int s = (int)(it % kLinStages);
        const uint32_t ph = (uint32_t)((it / kLinStages) & 1);
        if (!wait_bounded(bar_full + 8u * s, ph) || s_abort) {
          ok = false;
          break;
        }
        sm100::fence_after_sync();
        const uint32_t sa = sbase + (uint32_t)s * kLinStageBytes;
        const uint64_t da = sm100::desc_k_sw128(sa);
        const uint64_t db = sm100::desc_k_sw128(sa + Cfg::kABytes);
#pragma unroll
        for (int k = 0; k < kLinTileK / 16; ++k)   // 16 elements = 32 bytes per MMA
          sm100::mma_f16(d, da + (uint64_t)(2 * k), db + (uint64_t)(2 * k), idesc,
                         (kb | k) != 0 ? 1u : 0u);
        sm100::mma_commit(bar_empty + 8u * s);     // stage s is free once these complete
      }
      if (!ok) break;
      sm100::mma_commit(bar_accf + 8u * acc);      // accumulator ready for the epilogue
    }
    if (!ok) {
      s_abort = 1;
      record_failure(rk.state, rk.host_flag, kStatusLoadTimeout, call);
    }
    // every MMA issued has completed before tensor memory is released
    sm100::mma_commit(bar_drain);
    wait_bounded(bar_drain, 0u);
  } else if (warp >= 2) {
    // epilogue: tensor memory -> dtype -> staging -> owner's receive buffer
    const int q4 = warp & 3;                   // tensor-memory lane quarter of this warp
    const int et = (int)threadIdx.x - 64;      // 0..127
    const int row = q4 * 32 + lane;            // tile row this thread reads
    int64_t tc = 0;
    for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x, ++tc) {
      int64_t mb, nb;
      tile_mn(t, mb, nb);
      const int owner = (int)(nb / nbl);
      const int64_t nbo = nb - (int64_t)owner * nbl;
      const int acc = (int)(tc & 1);
      const uint32_t aph = (uint32_t)((tc >> 1) & 1);
      const bool ok = wait_bounded(bar_accf + 8u * acc, aph) && !s_abort;
      if (!ok) {
        s_abort = 1;
        record_failure(rk.state, rk.host_flag, kStatusLoadTimeout, call);
      }
      // every epilogue thread takes the same branch: s_abort is read after the barrier
      ptx::team_bar(1, 128);
      if (s_abort) break;
      sm100::fence_after_sync();
      unsigned char* srow = staging + (size_t)row * kLinPitch;
      // owner's partials [src = rank][row][col] of this tile
      unsigned char* dst = a.region[owner] + a.recv_off +
                           (((int64_t)rank * a.nmax + mb * kLinTileM) * hl + nbo * kBN) *
                               (int64_t)sizeof(T);
      constexpr int kCW = kBN < 128 ? kBN : 128;   // columns per pass through the staging
      constexpr int kChunks = kCW * 2 / 16;         // 16-byte chunks of a staged row
#pragma unroll 1
      for (int h = 0; h < kBN / kCW; ++h) {
#pragma unroll
        for (int c = 0; c < kCW / 32; ++c) {
          uint32_t r[32];
          sm100::tmem_ld_32x32(tmem + (uint32_t)(acc * kBN + h * kCW + c * 32) +
                                   ((uint32_t)(q4 * 32) << 16),
                               r);
          sm100::tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint4 v;
            v.x = pack2<T>(__uint_as_float(r[8 * j + 0]), __uint_as_float(r[8 * j + 1]));
            v.y = pack2<T>(__uint_as_float(r[8 * j + 2]), __uint_as_float(r[8 * j + 3]));
            v.z = pack2<T>(__uint_as_float(r[8 * j + 4]), __uint_as_float(r[8 * j + 5]));
            v.w = pack2<T>(__uint_as_float(r[8 * j + 6]), __uint_as_float(r[8 * j + 7]));
            *reinterpret_cast<uint4*>(srow + c * 64 + j * 16) = v;
          }
        }
        if (h == kBN / kCW - 1) {   // the whole accumulator has been read
          sm100::fence_before_sync();
          __syncwarp();
          if (lane == 0) ptx::mbar_arrive(bar_acce + 8u * acc);
        }
        ptx::team_bar(1, 128);   // staging complete
        // 128 rows x kCW * 2 bytes; a warp instruction stores whole rows of the pass
        // (2 rows x 256 contiguous bytes at 128 columns, 4 x 128 at 64)
        for (int idx = et; idx < kLinTileM * kChunks; idx += 128) {
          const int i = idx / kChunks, ch = idx % kChunks;
          if (mb * kLinTileM + i < a.rows) {
            const uint4 v =
                *reinterpret_cast<const uint4*>(staging + (size_t)i * kLinPitch + ch * 16);
            ptx::st_v4(dst + (int64_t)i * hl * (int64_t)sizeof(T) + h * kCW * 2 + ch * 16, v);
          }
        }
        ptx::team_bar(1, 128);   // every store issued (and the staging free)
      }
      if (et == 0) {
        __threadfence_system();   // the CTA's stores of the tile before its flag
        unsigned int* flag = reinterpret_cast<unsigned int*>(a.region[owner] + a.flags_off) +
                             (((int64_t)buf * tp + rank) * a.mblocks + mb) * a.nblocks + nbo;
        ptx::st_relaxed_sys_u32(flag, tag);
      }
    }
  }
  __syncthreads();   // phase 1 done on this CTA
  if (warp == 1) {
    sm100::fence_after_sync();
    sm100::tmem_dealloc(tmem, Cfg::kTmemCols);
  }

  // ------------------------------------------------------------------ phase 2
  // Rows [rows * c / G, rows * (c + 1) / G) of this rank's columns; warps take
  // rows round-robin. Pass A: x = sum of the tp partials in rank order,
  // z = x + residual, z -> out (scratch), this rank's sum of z^2 kept in its own
  // slot and pushed to every peer. Pass B: every rank's partial -> S, y from z.
  WaitStats ws;
  constexpr int kWarps = kLinThreads / 32;
  const int64_t r_lo = a.rows * (int64_t)blockIdx.x / gridDim.x;
  const int64_t r_hi = a.rows * ((int64_t)blockIdx.x + 1) / gridDim.x;
  const int V = (int)(hl * (int64_t)sizeof(T) / 16);          // 16-byte vectors per row
  unsigned char* outb = reinterpret_cast<unsigned char*>(rk.out);
  unsigned char* resb = reinterpret_cast<unsigned char*>(rk.res);
  const uint4* gam = reinterpret_cast<const uint4*>(rk.gamma);
  const unsigned char* recv = a.region[rank] + a.recv_off;
  const unsigned int* flags = reinterpret_cast<const unsigned int*>(a.region[rank] + a.flags_off);
  const unsigned long long* own = reinterpret_cast<const unsigned long long*>(a.region[rank]);
  const unsigned int* abort_flag = rk.state ? &rk.state->abort : nullptr;
  const int64_t row_bytes = hl * (int64_t)sizeof(T);
  bool ok = s_abort == 0;
  int64_t ready_mb = -1;
  for (int64_t i = r_lo + warp; i < r_hi && ok; i += kWarps) {
    const int64_t mb = i / kLinTileM;
    if (mb != ready_mb) {   // every rank's tiles of this 128-row block have landed
      const int nflags = tp * (int)a.nblocks;
      const unsigned long long t0 = ptx::globaltimer();
      for (unsigned n = 0;; ++n) {
        bool all = true;
        for (int f = lane; f < nflags; f += 32) {
          const int src = f / (int)a.nblocks, nbo = f - src * (int)a.nblocks;
          const unsigned int* fl =
              flags + (((int64_t)buf * tp + src) * a.mblocks + mb) * a.nblocks + nbo;
          if (ptx::ld_acquire_sys_u32(fl) != tag) all = false;
        }
        if (__all_sync(0xFFFFFFFFu, all)) break;
        bool give_up = false;
        if ((n & 7u) == 7u)
          give_up = ptx::globaltimer() - t0 > a.timeout_ns ||
                    (abort_flag && ptx::ld_relaxed_gpu_u32(abort_flag) != 0u);
        if (__any_sync(0xFFFFFFFFu, give_up)) {
          if (lane == 0) record_failure(rk.state, rk.host_flag, kStatusTimeout, call);
          ok = false;
          break;
        }
      }
      ready_mb = mb;
      if (!ok) break;
    }
    float ss = 0.f;
    for (int v = lane; v < V; v += 32) {
      float acc[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = 0.f;
      for (int src = 0; src < tp; ++src) {   // rank order: the same sum on every element
        const uint4 p =
            ptx::ld_stream_v4(recv + ((int64_t)src * a.nmax + i) * row_bytes + (int64_t)v * 16);
        float pf[8];
        Pack<T>::unpack(p, pf);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] += pf[e];
      }
      uint4 z = Pack<T>::pack(acc);                          // x, rounded to the dtype
      if (resb) {
        uint4* rv = reinterpret_cast<uint4*>(resb + i * row_bytes) + v;
        z = add16<T>(z, ptx::ld_stream_v4(rv));              // z = x + residual, rounded
        ptx::st_v4(rv, z);
      }
      ptx::st_v4(reinterpret_cast<uint4*>(outb + i * row_bytes) + v, z);
      ss += sumsq16<T>(z);
    }
    ss = warp_allreduce_sum(ss);
    if (lane < tp) {   // lane q: this rank's partial of row i into rank q's slot [buf][rank][i]
      unsigned long long* dst =
          reinterpret_cast<unsigned long long*>(a.region[lane]) + slot_index(buf, rank, tp, a.nmax, i);
      if (lane == rank)
        *reinterpret_cast<volatile unsigned long long*>(dst) = pack_slot(ss, tag);
      else
        store_slot(a.push_mode, dst, ss, tag);
    }
  }
  for (int64_t i = r_lo + warp; i < r_hi; i += kWarps) {
    // the same warp wrote row i in pass A (its own slot: program order)
    bool failed = !ok || s_abort != 0;
    float val = 0.f;
    if (lane < tp && !failed) {
      const unsigned long long* src = own + slot_index(buf, lane, tp, a.nmax, i);
      if (lane == rank) {
        val = slot_value(*reinterpret_cast<const volatile unsigned long long*>(src));
      } else {
        unsigned long long w = 0ull;
        const uint32_t f = wait_slot(a.push_mode, src, tag, a.timeout_ns, abort_flag, &w, ws);
        if (f == kStatusTimeout) record_failure(rk.state, rk.host_flag, kStatusTimeout, call);
        if (f != kStatusOk) failed = true;
        val = slot_value(w);
      }
    }
    failed = __any_sync(0xFFFFFFFFu, failed);
    float S = 0.f;
    for (int q = 0; q < tp; ++q) S += __shfl_sync(0xFFFFFFFFu, val, q);
    const float inv = failed ? quiet_nan() : rsqrtf(S / (float)a.hidden + a.eps);
    for (int v = lane; v < V; v += 32) {
      uint4* yv = reinterpret_cast<uint4*>(outb + i * row_bytes) + v;
      ptx::st_v4(yv, normalize16<T>(ptx::ld_stream_v4(yv), ptx::ld_cached_v4(gam + v), inv));
    }
  }
  if (exchange) finish_launch(rk.state, call);
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
LinearLayout linear_layout(int tp, int64_t nmax, int64_t hidden, int64_t base) {
  LinearLayout L{};
  L.mblocks = (nmax + kLinTileM - 1) / kLinTileM;
  L.nblocks = hidden / tp / kLinTileNMin;   // flags for the narrowest tiles (64 columns)
  L.flags_off = (base + 1023) & ~(int64_t)1023;
  const int64_t flag_bytes = 2 * (int64_t)tp * L.mblocks * L.nblocks * 4;
  L.recv_off = (L.flags_off + flag_bytes + 1023) & ~(int64_t)1023;
  L.bytes = L.recv_off + (int64_t)tp * nmax * (hidden / tp) * 2;
  return L;
}

namespace {
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link).
EncodeTiledFn encode_tiled(cudaError_t* err) {
  static std::once_flag once;
  static EncodeTiledFn fn = nullptr;
  static cudaError_t e0 = cudaSuccess;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    e0 = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (e0 == cudaSuccess && (q != cudaDriverEntryPointSuccess || p == nullptr))
      e0 = cudaErrorNotSupported;
    fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  *err = e0;
  return fn;
}

// Row-major [outer][inner] 16-bit matrix, boxes of box_outer rows x 64 elements
// (128 bytes, the 128-byte swizzle); zeros outside the matrix.
cudaError_t encode_2d(EncodeTiledFn fn, unsigned char* out, const void* base, int dtype,
                      uint64_t inner, uint64_t outer, uint32_t box_outer) {
  CUtensorMap* m = reinterpret_cast<CUtensorMap*>(out);
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {inner * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kLinTileK, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(m, dtype == kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                          : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                        2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

constexpr int kMaxDevices = 64;
std::atomic<int> g_lin_attr[kMaxDevices][2][3];

template <typename T>
const void* linear_kernel_of(int bn) {
  return bn == 256   ? reinterpret_cast<const void*>(tp_linear_rmsnorm_kernel<T, 256>)
         : bn == 128 ? reinterpret_cast<const void*>(tp_linear_rmsnorm_kernel<T, 128>)
                     : reinterpret_cast<const void*>(tp_linear_rmsnorm_kernel<T, 64>);
}
const void* linear_kernel(int dtype, int bn) {
  return dtype == kBF16 ? linear_kernel_of<__nv_bfloat16>(bn) : linear_kernel_of<__half>(bn);
}
uint32_t linear_smem(int bn) {
  return bn == 256 ? LinCfg<256>::kSmem : bn == 128 ? LinCfg<128>::kSmem : LinCfg<64>::kSmem;
}
}  // namespace

// Tile width of a call: the widest of 256 (when every owner's columns are whole
// 256-column tiles), 128 and 64 that still gives every SM a tile; 64 otherwise.
int linear_tile_width(int64_t rows, int64_t hidden, int64_t hl, int sms) {
  const int64_t mt = (rows + kLinTileM - 1) / kLinTileM;
  if (hl % 256 == 0 && mt * (hidden / 256) >= sms) return 256;
  if (mt * (hidden / 128) >= sms) return 128;
  return 64;
}
namespace {
}  // namespace

static_assert(sizeof(CUtensorMap) == 128, "a tensor map is 128 bytes");
static_assert(offsetof(LArgs, tmaps) % 64 == 0, "tensor maps 64-byte aligned in the parameters");

cudaError_t launch_linear(LArgs& a, const void* const* as, const void* const* ws, int dtype,
                          int device, int grid_y, cudaStream_t stream) {
  cudaError_t err = cudaSuccess;
  const EncodeTiledFn fn = encode_tiled(&err);
  if (err != cudaSuccess) return err;
  const int nranks = a.emulated ? grid_y : 1;
  int sms = 0;
  err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  if (err != cudaSuccess) return err;
  const int bn = linear_tile_width(a.rows, a.hidden, a.hl, sms / (grid_y > 1 ? grid_y : 1));
  a.nblocks = a.hl / bn;
  const uint32_t smem = linear_smem(bn);
  for (int r = 0; r < nranks; ++r) {
    err = encode_2d(fn, a.tmaps[2 * r], as[r], dtype, (uint64_t)a.k, (uint64_t)a.rows, kLinTileM);
    if (err != cudaSuccess) return err;
    err = encode_2d(fn, a.tmaps[2 * r + 1], ws[r], dtype, (uint64_t)a.k, (uint64_t)a.hidden,
                    (uint32_t)bn);
    if (err != cudaSuccess) return err;
  }
  const void* kfn = linear_kernel(dtype, bn);
  const int ti = dtype == kBF16 ? 0 : 1, bi = bn == 256 ? 2 : bn == 128 ? 1 : 0;
  const bool cacheable = device >= 0 && device < kMaxDevices;
  if (!cacheable || g_lin_attr[device][ti][bi].load() == 0) {
    err = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (err != cudaSuccess) return err;
    err = cudaFuncSetAttribute(kfn, cudaFuncAttributePreferredSharedMemoryCarveout,
                               (int)cudaSharedmemCarveoutMaxShared);
    if (err != cudaSuccess) return err;
    if (cacheable) g_lin_attr[device][ti][bi].store(1);
  }
  int per_sm = 0;
  err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kfn, kLinThreads, smem);
  if (err != cudaSuccess) return err;
  const int64_t resident = (int64_t)per_sm * sms / (grid_y > 1 ? grid_y : 1);
  const int64_t tiles = ((a.rows + kLinTileM - 1) / kLinTileM) * (a.hidden / bn);
  int64_t grid = tiles < resident ? tiles : resident;
  if (grid < 1) return cudaErrorCooperativeLaunchTooLarge;
  a.push_mode = get_push_mode();
  void* args[] = {&a};
  const dim3 g3((unsigned)grid, (unsigned)grid_y), blk(kLinThreads);
  if (grid_y > 1) return cudaLaunchCooperativeKernel(kfn, g3, blk, args, smem, stream);
  if (!get_dependent_launch()) return cudaLaunchKernel(kfn, g3, blk, args, smem, stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = g3;
  cfg.blockDim = blk;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelExC(&cfg, kfn, args);
}

}  // namespace rtp
