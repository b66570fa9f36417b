// Backward of the fused tensor-parallel RMSNorm for B200 (sm_100a).
//
// Forward (per row, rank k holding the columns of its slice):
//   S = sum over ranks of sum(x^2),  inv = rsqrt(S / hidden + eps),  y = x * inv * w.
// Backward, with g = dy * w:
//   D  = sum over ranks of sum(g * x)
//   dx = inv * g - x * (inv^3 * D / hidden)
//   dw = sum over rows of dy * x * inv          (the rank's own columns: no exchange)
// S and D are the only cross-rank quantities: one fp32 scalar each per row,
// exchanged through the forward's mailbox protocol in two consecutive
// generations (S with call g's tag in buffer g & 1, then D with call g + 1's
// tag in the other buffer), so a backward launch advances the generation by 2.
// A rank pushes a row's D only after it has received every peer's S of that
// row; hence when a rank has all of a call's D partials, every peer is done
// reading its S slots, and the next call may reuse that buffer.
//
// One CTA per row at a time (grid-stride over a grid of at most one resident
// wave), x, dy and w read with 16-byte loads when aligned (else per element);
// the second pass re-reads the row from L2. Each CTA accumulates its dw
// partial in shared memory (fp32) and writes it to its row of the workspace;
// a second kernel sums the partials in a fixed order (deterministic).
// No counterpart in the reference, which is forward-only.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>

#include "device_common.cuh"
#include "internal.h"
#include "ptx.cuh"
#include "rtp_common.h"

namespace rtp {

// kVec16: rows read as 16-byte chunks of Pack<T>::kE elements; else one element.
template <typename T, int kBlock, bool kVec16>
__global__ void __launch_bounds__(kBlock)
    tp_rmsnorm_backward_kernel(const __grid_constant__ BArgs b) {
  constexpr int kWarps = kBlock / 32;
  constexpr int kC = kVec16 ? Pack<T>::kE : 1;   // elements per chunk
  ptx::grid_dep_wait();
  ptx::grid_dep_launch_dependents();
  const KArgs& a = b.k;
  extern __shared__ float s_dw[];                // [hl]: this CTA's dw partial
  __shared__ float s_red[kWarps][2];
  __shared__ float s_tot[2];
  __shared__ int s_ok;
  __shared__ unsigned long long s_call;

  const unsigned long long t_start = a.prof ? ptx::globaltimer() : 0ull;
  WaitStats wst;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int ri = a.emulated ? (int)blockIdx.y : 0;
  const int rank = a.emulated ? (int)blockIdx.y : a.rank;
  const RankPtrs& rp = a.rp[ri];
  const T* __restrict__ xg = ptx::launder(reinterpret_cast<const T*>(rp.x));
  const T* __restrict__ wg = ptx::launder(reinterpret_cast<const T*>(rp.w));
  const T* __restrict__ dyg = ptx::launder(reinterpret_cast<const T*>(b.dy[ri]));
  T* __restrict__ dxg = reinterpret_cast<T*>(rp.out);
  const bool exchange = a.tp > 1;
  const int64_t hl = a.hl;
  const int64_t chunks = hl / kC;

  auto load = [&](const T* base, int64_t c, float (&f)[kC]) {
    if constexpr (kVec16) {
      Pack<T>::unpack(ptx::ld_cached_v4(reinterpret_cast<const uint4*>(base) + c), f);
    } else {
      f[0] = Pack<T>::to_f(base[c]);
    }
  };
  auto store = [&](T* base, int64_t c, const float (&f)[kC]) {
    if constexpr (kVec16) {
      ptx::st_v4(reinterpret_cast<uint4*>(base) + c, Pack<T>::pack(f));
    } else {
      base[c] = Pack<T>::from_f(f[0]);
    }
  };

  for (int64_t c = threadIdx.x; c < chunks; c += kBlock) {
#pragma unroll
    for (int e = 0; e < kC; ++e) s_dw[c * kC + e] = 0.f;
  }

  unsigned long long call = 0ull;
  uint32_t buf0 = 0u, tag0 = 0u, buf1 = 0u, tag1 = 0u;
  if (exchange) {
    if (threadIdx.x == 0) s_call = read_generation(rp.state);
    __syncthreads();
    call = s_call;
    buf0 = buffer_of(call);
    tag0 = tag_of(call);
    buf1 = buffer_of(call + 1ull);
    tag1 = tag_of(call + 1ull);
  }

  for (int64_t row = blockIdx.x; row < a.rows; row += gridDim.x) {
    const T* xr = xg + row * hl;
    const T* dyr = dyg + row * hl;
    // pass 1: local sum(x^2) and sum(dy * w * x)
    float s = 0.f, d = 0.f;
    for (int64_t c = threadIdx.x; c < chunks; c += kBlock) {
      float xf[kC], dyf[kC], wf[kC];
      load(xr, c, xf);
      load(dyr, c, dyf);
      load(wg, c, wf);
#pragma unroll
      for (int e = 0; e < kC; ++e) {
        s = fmaf(xf[e], xf[e], s);
        d = fmaf(dyf[e] * wf[e], xf[e], d);
      }
    }
    s = warp_allreduce_sum(s);
    d = warp_allreduce_sum(d);
    if (lane == 0) {
      s_red[warp][0] = s;
      s_red[warp][1] = d;
    }
    __syncthreads();
    if (warp == 0) {
      float S = 0.f, D = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        S += s_red[w][0];
        D += s_red[w][1];
      }
      bool ok = true;
      if (exchange) {
        // lane q < tp serves rank q: S first (generation `call`) ...
        bool failed = false;
        const float vs = push_poll(a, rank, rp, buf0, tag0, call, row, lane, lane < a.tp, S,
                                   failed, wst);
        ok = !__any_sync(0xFFFFFFFFu, failed);   // every lane's S poll ended before any D push
        float tot = 0.f;
        for (int p = 0; p < a.tp; ++p) tot += __shfl_sync(0xFFFFFFFFu, vs, p);
        S = tot;
        // ... then D (generation call + 1), rank order again
        failed = false;
        const float vd = push_poll(a, rank, rp, buf1, tag1, call + 1ull, row, lane, lane < a.tp, D,
                                   failed, wst);
        ok = !__any_sync(0xFFFFFFFFu, failed) && ok;
        tot = 0.f;
        for (int p = 0; p < a.tp; ++p) tot += __shfl_sync(0xFFFFFFFFu, vd, p);
        D = tot;
      }
      if (lane == 0) {
        s_tot[0] = S;
        s_tot[1] = D;
        s_ok = ok ? 1 : 0;
      }
    }
    __syncthreads();
    const float inv = s_ok ? rsqrtf(s_tot[0] / a.hidden_f + a.eps) : quiet_nan();
    const float coef = (inv * inv * inv) * (s_tot[1] / a.hidden_f);
    // pass 2 (x, dy, w again from L2): dx, and this CTA's dw partial
    T* dxr = dxg + row * hl;
    for (int64_t c = threadIdx.x; c < chunks; c += kBlock) {
      float xf[kC], dyf[kC], wf[kC], dxf[kC];
      load(xr, c, xf);
      load(dyr, c, dyf);
      load(wg, c, wf);
#pragma unroll
      for (int e = 0; e < kC; ++e) {
        dxf[e] = inv * (dyf[e] * wf[e]) - xf[e] * coef;
        s_dw[c * kC + e] += (dyf[e] * xf[e]) * inv;
      }
      store(dxr, c, dxf);
    }
    __syncthreads();   // s_red / s_tot are reused by the next row
  }

  // this CTA's dw partial -> its row of the workspace (each thread its own columns)
  float* wsr = b.ws[ri] + (int64_t)blockIdx.x * hl;
  for (int64_t c = threadIdx.x; c < chunks; c += kBlock) {
#pragma unroll
    for (int e = 0; e < kC; ++e) wsr[c * kC + e] = s_dw[c * kC + e];
  }
  if (exchange) finish_launch(rp.state, call, 2ull);
  flush_stats(a, wst, t_start);
}

// ---------------------------------------------------------------------------
// Register backward (aligned rows of up to 2048 16-byte vectors): the forward's
// teams and column mapping. A team of kW warps owns whole rows; lane l of warp
// wit holds the row's vectors c = (j * kW + wit) * 32 + l, j < kVec, of x and dy
// in registers, for kChunk rows at a time (all their loads in flight at once).
// Per chunk: S and D of every row in one pass (team reduction), the exchange
// (every row's S pushed, every S polled, then every D pushed and polled --
// a row's D is pushed only after its S exchange completed), then dx from the
// registers and dw accumulated per lane in fp32 registers (the lane's own
// columns, every row of the team). At the end the teams of a CTA add their dw
// partials into shared memory in team order, and the CTA writes its row of the
// workspace; backward_dw_reduce_kernel sums the rows in order (deterministic).
// x and dy are read once from HBM.
// ---------------------------------------------------------------------------
template <typename T, int kVec, int kW, int kBlock, int kMinBlocks, int kChunk>
__global__ void __launch_bounds__(kBlock, kMinBlocks)
    tp_rmsnorm_backward_vec_kernel(const __grid_constant__ BArgs b) {
  constexpr int kTeams = kBlock / 32 / kW;
  constexpr int kE = Pack<T>::kE;
  static_assert(kTeams >= 1 && kTeams <= 15, "team count must fit the named barriers");
  ptx::grid_dep_wait();
  ptx::grid_dep_launch_dependents();
  const KArgs& a = b.k;
  extern __shared__ float s_dw[];                    // [kTeams][hl]: each team's dw partial
  __shared__ float s_red[kTeams][kChunk][kW][2];
  __shared__ float s_tot[kTeams][kChunk][3];         // S, D, ok
  const unsigned long long t_start = a.prof ? ptx::globaltimer() : 0ull;
  WaitStats wst;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int team = warp / kW;
  const int wit = warp - team * kW;
  const int ri = a.emulated ? (int)blockIdx.y : 0;
  const int rank = a.emulated ? (int)blockIdx.y : a.rank;
  const RankPtrs& rp = a.rp[ri];
  const int64_t V = a.hl / kE;
  const uint4* __restrict__ xg = ptx::launder(reinterpret_cast<const uint4*>(rp.x));
  const uint4* __restrict__ wg = ptx::launder(reinterpret_cast<const uint4*>(rp.w));
  const uint4* __restrict__ dyg = ptx::launder(reinterpret_cast<const uint4*>(b.dy[ri]));
  uint4* __restrict__ dxg = reinterpret_cast<uint4*>(rp.out);
  const bool exchange = a.tp > 1;
  const int tp = a.tp;

  unsigned long long call = 0ull;
  uint32_t buf0 = 0u, tag0 = 0u, buf1 = 0u, tag1 = 0u;
  if (exchange) {
    call = read_generation(rp.state);
    buf0 = buffer_of(call);
    tag0 = tag_of(call);
    buf1 = buffer_of(call + 1ull);
    tag1 = tag_of(call + 1ull);
  }

  // this lane's columns of the team's dw partial (no other thread touches them)
  float* tdw = s_dw + (int64_t)team * a.hl;
#pragma unroll
  for (int j = 0; j < kVec; ++j) {
    const int c = (j * kW + wit) * 32 + lane;
    if (c < V) {
#pragma unroll
      for (int e = 0; e < kE; e += 4)
        *reinterpret_cast<float4*>(tdw + (int64_t)c * kE + e) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }

  const int64_t teams_total = (int64_t)gridDim.x * kTeams;
  const int64_t tg = (int64_t)blockIdx.x * kTeams + team;
  bool all_ok = true;
  // the team's rows: tg, tg + TT, tg + 2 TT, ... in chunks of kChunk
  for (int64_t base = tg; base < a.rows; base += (int64_t)kChunk * teams_total) {
    uint4 xv[kChunk][kVec], dv[kChunk][kVec];
#pragma unroll
    for (int i = 0; i < kChunk; ++i) {
      const int64_t row = base + i * teams_total;
#pragma unroll
      for (int j = 0; j < kVec; ++j) {
        const int c = (j * kW + wit) * 32 + lane;
        const bool in = row < a.rows && c < V;
        xv[i][j] = in ? ptx::ld_stream_v4(xg + row * V + c) : make_uint4(0u, 0u, 0u, 0u);
        dv[i][j] = in ? ptx::ld_stream_v4(dyg + row * V + c) : make_uint4(0u, 0u, 0u, 0u);
      }
    }
    // S = sum x^2 and D = sum dy * w * x of every row of the chunk
    float S[kChunk], D[kChunk];
#pragma unroll
    for (int i = 0; i < kChunk; ++i) {
      float s = 0.f, d = 0.f;
#pragma unroll
      for (int j = 0; j < kVec; ++j) {
        const int c = (j * kW + wit) * 32 + lane;
        if (c < V) {
          float xf[kE], df[kE], wf[kE];
          Pack<T>::unpack(xv[i][j], xf);
          Pack<T>::unpack(dv[i][j], df);
          Pack<T>::unpack(ptx::ld_cached_v4(wg + c), wf);
#pragma unroll
          for (int e = 0; e < kE; ++e) {
            s = fmaf(xf[e], xf[e], s);
            d = fmaf(df[e] * wf[e], xf[e], d);
          }
        }
      }
      S[i] = warp_allreduce_sum(s);
      D[i] = warp_allreduce_sum(d);
    }
    if constexpr (kW > 1) {
      if (lane == 0) {
#pragma unroll
        for (int i = 0; i < kChunk; ++i) {
          s_red[team][i][wit][0] = S[i];
          s_red[team][i][wit][1] = D[i];
        }
      }
      ptx::team_bar(1 + team, kW * 32);
#pragma unroll
      for (int i = 0; i < kChunk; ++i) {
        float s = 0.f, d = 0.f;
#pragma unroll
        for (int w = 0; w < kW; ++w) {
          s += s_red[team][i][w][0];
          d += s_red[team][i][w][1];
        }
        S[i] = s;
        D[i] = d;
      }
    }
    bool ok[kChunk];
#pragma unroll
    for (int i = 0; i < kChunk; ++i) ok[i] = true;
    if (exchange) {
      if (kW == 1 || wit == 0) {
        // lane q < tp serves rank q: every row's S, then every row's D
        const bool lq = lane < tp;
#pragma unroll
        for (int i = 0; i < kChunk; ++i) {
          const int64_t row = base + i * teams_total;
          push_slot(a, rank, buf0, tag0, row, lane, lq && row < a.rows, S[i]);
        }
#pragma unroll
        for (int i = 0; i < kChunk; ++i) {
          const int64_t row = base + i * teams_total;
          bool failed = false;
          const float v = poll_slot(a, rank, rp, buf0, tag0, call, row, lane, lq && row < a.rows,
                                    S[i], failed, wst);
          ok[i] = !__any_sync(0xFFFFFFFFu, failed);   // every S poll ended before any D push
          float t = 0.f;
          for (int p = 0; p < tp; ++p) t += __shfl_sync(0xFFFFFFFFu, v, p);
          S[i] = t;
        }
#pragma unroll
        for (int i = 0; i < kChunk; ++i) {
          const int64_t row = base + i * teams_total;
          push_slot(a, rank, buf1, tag1, row, lane, lq && row < a.rows, D[i]);
        }
#pragma unroll
        for (int i = 0; i < kChunk; ++i) {
          const int64_t row = base + i * teams_total;
          bool failed = false;
          const float v = poll_slot(a, rank, rp, buf1, tag1, call + 1ull, row, lane,
                                    lq && row < a.rows, D[i], failed, wst);
          ok[i] = !__any_sync(0xFFFFFFFFu, failed) && ok[i];
          float t = 0.f;
          for (int p = 0; p < tp; ++p) t += __shfl_sync(0xFFFFFFFFu, v, p);
          D[i] = t;
        }
      }
      if constexpr (kW > 1) {
        if (wit == 0 && lane == 0) {
#pragma unroll
          for (int i = 0; i < kChunk; ++i) {
            s_tot[team][i][0] = S[i];
            s_tot[team][i][1] = D[i];
            s_tot[team][i][2] = ok[i] ? 1.f : 0.f;
          }
        }
        ptx::team_bar(1 + team, kW * 32);
#pragma unroll
        for (int i = 0; i < kChunk; ++i) {
          S[i] = s_tot[team][i][0];
          D[i] = s_tot[team][i][1];
          ok[i] = s_tot[team][i][2] != 0.f;
        }
      }
    }
    // dx from the registers; dw partial of the lane's columns
#pragma unroll
    for (int i = 0; i < kChunk; ++i) {
      const int64_t row = base + i * teams_total;
      if (row >= a.rows) break;
      if (!ok[i]) all_ok = false;
      const float inv = ok[i] ? rsqrtf(S[i] / a.hidden_f + a.eps) : quiet_nan();
      const float coef = (inv * inv * inv) * (D[i] / a.hidden_f);
#pragma unroll
      for (int j = 0; j < kVec; ++j) {
        const int c = (j * kW + wit) * 32 + lane;
        if (c < V) {
          float xf[kE], df[kE], wf[kE], o[kE];
          Pack<T>::unpack(xv[i][j], xf);
          Pack<T>::unpack(dv[i][j], df);
          Pack<T>::unpack(ptx::ld_cached_v4(wg + c), wf);
          float* dwp = tdw + (int64_t)c * kE;
#pragma unroll
          for (int e = 0; e < kE; e += 4) {
            float4 acc = *reinterpret_cast<float4*>(dwp + e);
            acc.x += (df[e + 0] * xf[e + 0]) * inv;
            acc.y += (df[e + 1] * xf[e + 1]) * inv;
            acc.z += (df[e + 2] * xf[e + 2]) * inv;
            acc.w += (df[e + 3] * xf[e + 3]) * inv;
            *reinterpret_cast<float4*>(dwp + e) = acc;
          }
#pragma unroll
          for (int e = 0; e < kE; ++e) o[e] = inv * (df[e] * wf[e]) - xf[e] * coef;
          ptx::st_v4(dxg + row * V + c, Pack<T>::pack(o));
        }
      }
    }
  }
  (void)all_ok;
  // the CTA's row of the workspace: the teams' partials added in team order
  __syncthreads();
  float* wsr = b.ws[ri] + (int64_t)blockIdx.x * a.hl;
  for (int64_t i = threadIdx.x; i < a.hl; i += kBlock) {
    float acc = s_dw[i];
#pragma unroll
    for (int t = 1; t < kTeams; ++t) acc += s_dw[(int64_t)t * a.hl + i];
    wsr[i] = acc;
  }
  if (exchange) finish_launch(rp.state, call, 2ull);
  flush_stats(a, wst, t_start);
}

// ---------------------------------------------------------------------------
// Local ring backward (TP = 1, aligned rows; the default there): the register
// backward's teams, rows and column mapping, but a team's rows of x and dy are
// staged in shared memory by bulk copies -- kStages stages per team, a row's x
// and dy on one mbarrier -- and each thread accumulates dw for its columns in
// registers. With the row buffers out of the registers, kStages - 1 rows per
// team are in flight while one is processed (the bytes in flight per SM are
// set by shared memory), and dw needs no shared-memory read-modify-write per
// row. A stage is refilled once every thread of the team is past the team
// barrier of the following row. At the end the teams' dw registers are summed
// in team order through shared memory into the CTA's fp32 part of the
// workspace, as in the register kernels.
// ---------------------------------------------------------------------------
template <typename T, int kVec, int kW, int kBlock, int kStages>
__global__ void __launch_bounds__(kBlock, 512 / kBlock)
    rmsnorm_local_backward_ring_kernel(const __grid_constant__ BArgs b) {
  constexpr int kTeams = kBlock / 32 / kW;
  constexpr int kE = Pack<T>::kE;
  static_assert(kTeams >= 1 && kTeams <= 15, "team count must fit the named barriers");
  static_assert(kStages >= 2, "one stage in use, at least one in flight");
  ptx::grid_dep_wait();
  ptx::grid_dep_launch_dependents();
  const KArgs& a = b.k;
  extern __shared__ __align__(128) unsigned char smem[];   // [kTeams][kStages][x row | dy row]
  __shared__ __align__(8) unsigned long long s_bar[kTeams][kStages];
  __shared__ float s_red[kTeams][2][kW][2];
  __shared__ int s_ok[kTeams][2][kW];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int team = warp / kW;
  const int wit = warp - team * kW;
  const RankPtrs& rp = a.rp[0];
  const int64_t V = a.hl / kE;
  const uint32_t row_bytes = (uint32_t)V * 16u;
  const uint32_t stage_bytes = 2u * row_bytes;
  const uint32_t ring_addr = ptx::smem_addr(smem) + (uint32_t)team * kStages * stage_bytes;
  const unsigned char* ring = smem + (size_t)team * kStages * stage_bytes;
  const uint32_t bar0 = ptx::smem_addr(&s_bar[team][0]);
  const unsigned char* xg = reinterpret_cast<const unsigned char*>(rp.x);
  const unsigned char* dyg = reinterpret_cast<const unsigned char*>(b.dy[0]);
  const uint4* __restrict__ wg = ptx::launder(reinterpret_cast<const uint4*>(rp.w));
  uint4* dxg = reinterpret_cast<uint4*>(rp.out);
  const int64_t teams_total = (int64_t)gridDim.x * kTeams;
  const int64_t tg = (int64_t)blockIdx.x * kTeams + team;
  const int64_t my_rows = tg < a.rows ? (a.rows - 1 - tg) / teams_total + 1 : 0;
  const bool producer = wit == 0 && lane == 0;

  auto issue = [&](int64_t kk) {   // the team's kk-th row -> stage kk % kStages
    const uint32_t st = (uint32_t)(kk % kStages);
    const int64_t row = tg + kk * teams_total;
    const uint32_t bar = bar0 + 8u * st;
    ptx::mbar_arrive_expect_tx(bar, stage_bytes);
    ptx::bulk_load(ring_addr + st * stage_bytes, xg + row * (int64_t)row_bytes, row_bytes, bar);
    ptx::bulk_load(ring_addr + st * stage_bytes + row_bytes, dyg + row * (int64_t)row_bytes,
                   row_bytes, bar);
  };
  int64_t issued = my_rows < kStages ? my_rows : kStages;
  if (producer) {
#pragma unroll
    for (int st = 0; st < kStages; ++st) ptx::mbar_init(bar0 + 8u * st, 1u);
    ptx::fence_mbar_init();
    for (int64_t kk = 0; kk < issued; ++kk) issue(kk);
  }
  // this thread's weight vectors, and its dw columns' accumulators
  uint4 wv[kVec];
  float dw[kVec][kE];
#pragma unroll
  for (int j = 0; j < kVec; ++j) {
    const int c = (j * kW + wit) * 32 + lane;
    wv[j] = c < V ? ptx::ld_cached_v4(wg + c) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
    for (int e = 0; e < kE; ++e) dw[j][e] = 0.f;
  }
  if constexpr (kW > 1)
    ptx::team_bar(1 + team, kW * 32);   // the barriers' initialisation, before any wait
  else
    __syncwarp();

  bool load_ok = true;
  int64_t k = 0;
  for (; k < my_rows; ++k) {
    const int slot = (int)(k & 1);
    const uint32_t st = (uint32_t)(k % kStages);
    bool ok = mbar_wait_bounded(bar0 + 8u * st, (uint32_t)((k / kStages) & 1), kLoadTimeoutNs);
    const uint4* xs = reinterpret_cast<const uint4*>(ring + (size_t)st * stage_bytes);
    const uint4* ds = reinterpret_cast<const uint4*>(ring + (size_t)st * stage_bytes + row_bytes);
    float s = 0.f, d = 0.f;
#pragma unroll
    for (int j = 0; j < kVec; ++j) {
      const int c = (j * kW + wit) * 32 + lane;
      const bool in = ok && c < V;
      float xf[kE], df[kE], wf[kE];
      Pack<T>::unpack(in ? xs[c] : make_uint4(0u, 0u, 0u, 0u), xf);
      Pack<T>::unpack(in ? ds[c] : make_uint4(0u, 0u, 0u, 0u), df);
      Pack<T>::unpack(wv[j], wf);
#pragma unroll
      for (int e = 0; e < kE; ++e) {
        s = fmaf(xf[e], xf[e], s);
        d = fmaf(df[e] * wf[e], xf[e], d);
      }
    }
    float S = warp_allreduce_sum(s), D = warp_allreduce_sum(d);
    ok = __all_sync(0xFFFFFFFFu, ok);
    if constexpr (kW > 1) {
      if (lane == 0) {
        s_red[team][slot][wit][0] = S;
        s_red[team][slot][wit][1] = D;
        s_ok[team][slot][wit] = ok ? 1 : 0;
      }
      ptx::team_bar(1 + team, kW * 32);
      S = 0.f;
      D = 0.f;
#pragma unroll
      for (int w = 0; w < kW; ++w) {
        S += s_red[team][slot][w][0];
        D += s_red[team][slot][w][1];
        ok = ok && s_ok[team][slot][w] != 0;
      }
    } else {
      __syncwarp();
    }
    if (!ok) {   // uniform over the team
      load_ok = false;
      break;
    }
    // every thread of the team is past its reads of the previous row's stage
    if (producer && k >= 1 && k - 1 + kStages < my_rows) {
      ptx::fence_proxy_async_smem();
      issue(k - 1 + kStages);
      ++issued;
    }
    const int64_t row = tg + k * teams_total;
    const float inv = rsqrtf(S / a.hidden_f + a.eps);
    const float coef = (inv * inv * inv) * (D / a.hidden_f);
    // x and dy read from the stage again (it is refilled only after the next
    // row's team barrier): fewer live registers than keeping them
#pragma unroll
    for (int j = 0; j < kVec; ++j) {
      const int c = (j * kW + wit) * 32 + lane;
      if (c < V) {
        float xf[kE], df[kE], wf[kE], o[kE];
        Pack<T>::unpack(xs[c], xf);
        Pack<T>::unpack(ds[c], df);
        Pack<T>::unpack(wv[j], wf);
#pragma unroll
        for (int e = 0; e < kE; ++e) {
          dw[j][e] += (df[e] * xf[e]) * inv;
          o[e] = inv * (df[e] * wf[e]) - xf[e] * coef;
        }
        ptx::st_v4(dxg + row * V + c, Pack<T>::pack(o));
      }
    }
  }
  if (!load_ok && producer) {
    // a copy never landed: wait (bounded) for the copies still in flight, so
    // none lands in shared memory that this CTA no longer owns
    for (int64_t kk = k; kk < issued; ++kk)
      mbar_wait_bounded(bar0 + 8u * (uint32_t)(kk % kStages), (uint32_t)((kk / kStages) & 1),
                        kLoadTimeoutNs);
  }
  __syncthreads();   // every stage read and every copy landed: the ring becomes [kTeams][hl] fp32
  float* s_dw = reinterpret_cast<float*>(smem);
  float* tdw = s_dw + (int64_t)team * a.hl;
#pragma unroll
  for (int j = 0; j < kVec; ++j) {
    const int c = (j * kW + wit) * 32 + lane;
    if (c < V) {
#pragma unroll
      for (int e = 0; e < kE; e += 4)
        *reinterpret_cast<float4*>(tdw + (int64_t)c * kE + e) =
            make_float4(dw[j][e], dw[j][e + 1], dw[j][e + 2], dw[j][e + 3]);
    }
  }
  __syncthreads();
  float* wsr = b.ws[0] + (int64_t)blockIdx.x * a.hl;
  for (int64_t i = threadIdx.x; i < a.hl; i += kBlock) {
    float acc = s_dw[i];
#pragma unroll
    for (int t = 1; t < kTeams; ++t) acc += s_dw[(int64_t)t * a.hl + i];
    wsr[i] = acc;
  }
}

// ---------------------------------------------------------------------------
// Local register backward (TP = 1: no exchange): the register backward's teams,
// column mapping and dw slices, one row at a time but double-buffered -- the
// next row's x and dy loads are issued before the current row is reduced,
// written and accumulated, so HBM stays busy through the compute and the dx
// stores (the chunked kernel above waits for each chunk's loads after the
// previous chunk's stores).
// ---------------------------------------------------------------------------
template <typename T, int kVec, int kW, int kBlock, int kMinBlocks>
__global__ void __launch_bounds__(kBlock, kMinBlocks)
    rmsnorm_local_backward_vec_kernel(const __grid_constant__ BArgs b) {
  constexpr int kTeams = kBlock / 32 / kW;
  constexpr int kE = Pack<T>::kE;
  static_assert(kTeams >= 1 && kTeams <= 15, "team count must fit the named barriers");
  ptx::grid_dep_wait();
  ptx::grid_dep_launch_dependents();
  const KArgs& a = b.k;
  extern __shared__ float s_dw[];                    // [kTeams][hl]: each team's dw partial
  __shared__ float s_red[kTeams][2][kW][2];          // two slots: rows alternate
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int team = warp / kW;
  const int wit = warp - team * kW;
  const RankPtrs& rp = a.rp[0];
  const int64_t V = a.hl / kE;
  const uint4* __restrict__ xg = ptx::launder(reinterpret_cast<const uint4*>(rp.x));
  const uint4* __restrict__ wg = ptx::launder(reinterpret_cast<const uint4*>(rp.w));
  const uint4* __restrict__ dyg = ptx::launder(reinterpret_cast<const uint4*>(b.dy[0]));
  uint4* __restrict__ dxg = reinterpret_cast<uint4*>(rp.out);

  float* tdw = s_dw + (int64_t)team * a.hl;
#pragma unroll
  for (int j = 0; j < kVec; ++j) {
    const int c = (j * kW + wit) * 32 + lane;
    if (c < V) {
#pragma unroll
      for (int e = 0; e < kE; e += 4)
        *reinterpret_cast<float4*>(tdw + (int64_t)c * kE + e) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }

  auto load = [&](int64_t row, uint4 (&xv)[kVec], uint4 (&dv)[kVec]) {
#pragma unroll
    for (int j = 0; j < kVec; ++j) {
      const int c = (j * kW + wit) * 32 + lane;
      const bool in = c < V;
      xv[j] = in ? ptx::ld_stream_v4(xg + row * V + c) : make_uint4(0u, 0u, 0u, 0u);
      dv[j] = in ? ptx::ld_stream_v4(dyg + row * V + c) : make_uint4(0u, 0u, 0u, 0u);
    }
  };
  // S, D (team), dx from the registers, dw into the team's slice
  auto process = [&](int64_t row, const uint4 (&xv)[kVec], const uint4 (&dv)[kVec], int slot) {
    float s = 0.f, d = 0.f;
#pragma unroll
    for (int j = 0; j < kVec; ++j) {
      const int c = (j * kW + wit) * 32 + lane;
      if (c < V) {
        float xf[kE], df[kE], wf[kE];
        Pack<T>::unpack(xv[j], xf);
        Pack<T>::unpack(dv[j], df);
        Pack<T>::unpack(ptx::ld_cached_v4(wg + c), wf);
#pragma unroll
        for (int e = 0; e < kE; ++e) {
          s = fmaf(xf[e], xf[e], s);
          d = fmaf(df[e] * wf[e], xf[e], d);
        }
      }
    }
    float S = warp_allreduce_sum(s), D = warp_allreduce_sum(d);
    if constexpr (kW > 1) {
      if (lane == 0) {
        s_red[team][slot][wit][0] = S;
        s_red[team][slot][wit][1] = D;
      }
      ptx::team_bar(1 + team, kW * 32);
      S = 0.f;
      D = 0.f;
#pragma unroll
      for (int w = 0; w < kW; ++w) {
        S += s_red[team][slot][w][0];
        D += s_red[team][slot][w][1];
      }
    }
    const float inv = rsqrtf(S / a.hidden_f + a.eps);
    const float coef = (inv * inv * inv) * (D / a.hidden_f);
#pragma unroll
    for (int j = 0; j < kVec; ++j) {
      const int c = (j * kW + wit) * 32 + lane;
      if (c < V) {
        float xf[kE], df[kE], wf[kE], o[kE];
        Pack<T>::unpack(xv[j], xf);
        Pack<T>::unpack(dv[j], df);
        Pack<T>::unpack(ptx::ld_cached_v4(wg + c), wf);
        float* dwp = tdw + (int64_t)c * kE;
#pragma unroll
        for (int e = 0; e < kE; e += 4) {
          float4 acc = *reinterpret_cast<float4*>(dwp + e);
          acc.x += (df[e + 0] * xf[e + 0]) * inv;
          acc.y += (df[e + 1] * xf[e + 1]) * inv;
          acc.z += (df[e + 2] * xf[e + 2]) * inv;
          acc.w += (df[e + 3] * xf[e + 3]) * inv;
          *reinterpret_cast<float4*>(dwp + e) = acc;
        }
#pragma unroll
        for (int e = 0; e < kE; ++e) o[e] = inv * (df[e] * wf[e]) - xf[e] * coef;
        ptx::st_v4(dxg + row * V + c, Pack<T>::pack(o));
      }
    }
  };

  const int64_t teams_total = (int64_t)gridDim.x * kTeams;
  int64_t row = (int64_t)blockIdx.x * kTeams + team;
  uint4 xa[kVec], da[kVec], xb[kVec], db[kVec];
  if (row < a.rows) load(row, xa, da);
  while (row < a.rows) {
    int64_t nxt = row + teams_total;
    if (nxt < a.rows) load(nxt, xb, db);
    process(row, xa, da, 0);
    row = nxt;
    if (row >= a.rows) break;
    nxt = row + teams_total;
    if (nxt < a.rows) load(nxt, xa, da);
    process(row, xb, db, 1);
    row = nxt;
  }
  __syncthreads();
  float* wsr = b.ws[0] + (int64_t)blockIdx.x * a.hl;
  for (int64_t i = threadIdx.x; i < a.hl; i += kBlock) {
    float acc = s_dw[i];
#pragma unroll
    for (int t = 1; t < kTeams; ++t) acc += s_dw[(int64_t)t * a.hl + i];
    wsr[i] = acc;
  }
}

// dw[j] = sum over the parts of ws[part][j]: a CTA takes 32 columns; its 16 warps
// each sum a contiguous range of parts (lane = column, coalesced), and warp 0
// adds the 16 range sums in range order -- the same order on every call.
constexpr int kDwWarps = 16;
constexpr int kDwMaxPer = (kBackwardMaxGrid + kDwWarps - 1) / kDwWarps;

template <typename T>
__global__ void __launch_bounds__(kDwWarps * 32)
    backward_dw_reduce_kernel(const float* __restrict__ ws, int parts, int64_t hl,
                              T* __restrict__ dw) {
  __shared__ float s_part[kDwWarps][32];
  ptx::grid_dep_wait();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t j = (int64_t)blockIdx.x * 32 + lane;
  const int per = (parts + kDwWarps - 1) / kDwWarps;
  const int c0 = warp * per, c1 = min(parts, c0 + per);
  // every load of the range in flight before the first add (one L2 round trip
  // instead of one per part); the adds then run in part order
  float v[kDwMaxPer];
#pragma unroll
  for (int i = 0; i < kDwMaxPer; ++i)
    v[i] = (j < hl && c0 + i < c1) ? ws[(int64_t)(c0 + i) * hl + j] : 0.f;
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kDwMaxPer; ++i) s += v[i];
  s_part[warp][lane] = s;
  __syncthreads();
  if (warp == 0 && j < hl) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < kDwWarps; ++w) t += s_part[w][lane];
    dw[j] = Pack<T>::from_f(t);
  }
}

namespace {

constexpr int kBwdBlock = 256;
using BwdFn = void (*)(const BArgs);

BwdFn backward_fn(int dtype, bool vec16) {
  switch (dtype) {
    case kF32:
      return vec16 ? tp_rmsnorm_backward_kernel<float, kBwdBlock, true>
                   : tp_rmsnorm_backward_kernel<float, kBwdBlock, false>;
    case kBF16:
      return vec16 ? tp_rmsnorm_backward_kernel<__nv_bfloat16, kBwdBlock, true>
                   : tp_rmsnorm_backward_kernel<__nv_bfloat16, kBwdBlock, false>;
    default:
      return vec16 ? tp_rmsnorm_backward_kernel<__half, kBwdBlock, true>
                   : tp_rmsnorm_backward_kernel<__half, kBwdBlock, false>;
  }
}

constexpr int kMaxDevices = 64;
std::atomic<unsigned int> g_smem_set[kMaxDevices][3][2];   // max dynamic smem raised to this

// Register backward shapes by 16-byte vectors per row V: the first whose capacity
// 32 * kW * kVec >= V (kVec, kW, block, CTAs per SM), two rows in flight per team.
struct BwdShape {
  int vec, w, block;
};
constexpr BwdShape kBwdShapes[] = {{1, 1, 256}, {2, 1, 256}, {4, 1, 256}, {4, 2, 256},
                                   {4, 4, 256}, {4, 8, 256}, {4, 16, 512}};
constexpr int kNumBwdShapes = sizeof(kBwdShapes) / sizeof(kBwdShapes[0]);
// rows in flight per team (x and dy of each in registers; dw lives in shared memory)
template <typename T, int kVec>
constexpr int bwd_chunk() {
  return 2;
}

template <typename T>
struct BwdVecTable {
#define RTP_BWD(V, W, B, M) tp_rmsnorm_backward_vec_kernel<T, V, W, B, M, bwd_chunk<T, V>()>
  static constexpr BwdFn fn[kNumBwdShapes] = {
      RTP_BWD(1, 1, 256, 2), RTP_BWD(2, 1, 256, 2), RTP_BWD(4, 1, 256, 2), RTP_BWD(4, 2, 256, 2),
      RTP_BWD(4, 4, 256, 2), RTP_BWD(4, 8, 256, 2), RTP_BWD(4, 16, 512, 1),
  };
#undef RTP_BWD
};

template <typename T>
struct BwdLocalTable {
#define RTP_BWDL(V, W, B, M) rmsnorm_local_backward_vec_kernel<T, V, W, B, M>
  static constexpr BwdFn fn[kNumBwdShapes] = {
      RTP_BWDL(1, 1, 256, 2), RTP_BWDL(2, 1, 256, 2), RTP_BWDL(4, 1, 256, 2), RTP_BWDL(4, 2, 256, 2),
      RTP_BWDL(4, 4, 256, 2), RTP_BWDL(4, 8, 256, 2), RTP_BWDL(4, 16, 512, 1),
  };
#undef RTP_BWDL
};

// the ring kernel: the same (vec, w) shapes and blocks; three stages per team,
// so a CTA's ring is at most 96 KB (two CTAs per SM), 192 KB for the last shape
// (one 512-thread team, one CTA per SM). (512-thread CTAs for every shape of two
// or more warps per team, one dw part per SM, measured no faster on B200: bf16
// 4096 x 4096, 22.3 us against 21.6 us.)
constexpr int kBwdRingStages = 3;
constexpr int kBwdRingBlock[kNumBwdShapes] = {256, 256, 256, 256, 256, 256, 512};
// below this many rows the register kernel's shorter start wins
constexpr int64_t kBwdRingMinRows = 1024;
template <typename T>
struct BwdRingTable {
#define RTP_BWDR(V, W, I) rmsnorm_local_backward_ring_kernel<T, V, W, kBwdRingBlock[I], kBwdRingStages>
  static constexpr BwdFn fn[kNumBwdShapes] = {
      RTP_BWDR(1, 1, 0), RTP_BWDR(2, 1, 1), RTP_BWDR(4, 1, 2), RTP_BWDR(4, 2, 3),
      RTP_BWDR(4, 4, 4), RTP_BWDR(4, 8, 5), RTP_BWDR(4, 16, 6),
  };
#undef RTP_BWDR
};

BwdFn backward_ring_fn(int dtype, int shape) {
  switch (dtype) {
    case kF32:
      return BwdRingTable<float>::fn[shape];
    case kBF16:
      return BwdRingTable<__nv_bfloat16>::fn[shape];
    default:
      return BwdRingTable<__half>::fn[shape];
  }
}

BwdFn backward_local_fn(int dtype, int shape) {
  switch (dtype) {
    case kF32:
      return BwdLocalTable<float>::fn[shape];
    case kBF16:
      return BwdLocalTable<__nv_bfloat16>::fn[shape];
    default:
      return BwdLocalTable<__half>::fn[shape];
  }
}

BwdFn backward_vec_fn(int dtype, int shape) {
  switch (dtype) {
    case kF32:
      return BwdVecTable<float>::fn[shape];
    case kBF16:
      return BwdVecTable<__nv_bfloat16>::fn[shape];
    default:
      return BwdVecTable<__half>::fn[shape];
  }
}
std::atomic<unsigned int> g_vec_smem_set[kMaxDevices][3][kNumBwdShapes];
std::atomic<unsigned int> g_local_smem_set[kMaxDevices][3][kNumBwdShapes];
std::atomic<unsigned int> g_ring_smem_set[kMaxDevices][3][kNumBwdShapes];

}  // namespace

cudaError_t launch_backward(const BArgs& b, int dtype, int device, int grid_y, cudaStream_t stream,
                            int* grid_out) {
  const KArgs& a = b.k;
  const int nranks = a.emulated ? grid_y : 1;
  const int eb = elem_bytes(dtype);
  bool vec16 = (a.hl * eb) % 16 == 0;
  for (int r = 0; r < nranks; ++r) {
    const uintptr_t bits = reinterpret_cast<uintptr_t>(a.rp[r].x) |
                           reinterpret_cast<uintptr_t>(a.rp[r].out) |
                           reinterpret_cast<uintptr_t>(a.rp[r].w) |
                           reinterpret_cast<uintptr_t>(b.dy[r]);
    if (bits & 15u) vec16 = false;
  }
  // the register kernel for aligned rows of up to 2048 vectors (unless the
  // bulk family is forced, which keeps the one-CTA-per-row kernel for comparison)
  const int64_t V = vec16 ? a.hl * eb / 16 : 0;
  int shape = -1;
  if (vec16 && get_family() != kFamilyBulk)
    for (int i = 0; i < kNumBwdShapes && shape < 0; ++i)
      if (V <= 32ll * kBwdShapes[i].w * kBwdShapes[i].vec) shape = i;
  // TP = 1 (no exchange): the ring kernel (bulk copies of x and dy into shared
  // memory), or with the register family forced the double-buffered register kernel
  const bool local = shape >= 0 && a.tp == 1 && !a.emulated;
  const bool ring = local && get_family() != kFamilyRegister && a.rows >= kBwdRingMinRows;
  const BwdFn fn = ring    ? backward_ring_fn(dtype, shape)
                   : local ? backward_local_fn(dtype, shape)
                   : shape >= 0 ? backward_vec_fn(dtype, shape) : backward_fn(dtype, vec16);
  const int block = ring ? kBwdRingBlock[shape] : shape >= 0 ? kBwdShapes[shape].block : kBwdBlock;
  const void* fp = reinterpret_cast<const void*>(fn);
  // dw partials: one [hl] fp32 slice per team (register kernels) or per CTA; the
  // ring kernel's shared memory is its stages (which later hold the slices)
  const int teams = shape >= 0 ? block / 32 / kBwdShapes[shape].w : 1;
  size_t smem = (size_t)teams * (size_t)a.hl * sizeof(float);
  if (ring) {
    const size_t stages = (size_t)teams * kBwdRingStages * 2u * (size_t)V * 16u;
    if (stages > smem) smem = stages;
  }
  cudaError_t err;
  // the 48 KB default limit counts static shared memory too: raise it early
  if (smem > 32u * 1024u) {
    const bool cacheable = device >= 0 && device < kMaxDevices;
    std::atomic<unsigned int>& set = ring         ? g_ring_smem_set[device][dtype][shape]
                                     : local      ? g_local_smem_set[device][dtype][shape]
                                     : shape >= 0 ? g_vec_smem_set[device][dtype][shape]
                                                  : g_smem_set[device][dtype][vec16 ? 1 : 0];
    if (!cacheable || set.load() < smem) {
      err = cudaFuncSetAttribute(fp, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (err != cudaSuccess) return err;
      if (cacheable) set.store((unsigned)smem);
    }
  }
  int per_sm = 0, sms = 0;
  err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fp, block, smem);
  if (err != cudaSuccess) return err;
  err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  if (err != cudaSuccess) return err;
  int64_t grid = (int64_t)per_sm * sms / (grid_y > 1 ? grid_y : 1);   // one resident wave
  if (grid > kBackwardMaxGrid) grid = kBackwardMaxGrid;
  if (grid > a.rows) grid = a.rows;
  if (grid < 1) return cudaErrorCooperativeLaunchTooLarge;
  if (grid_out) *grid_out = (int)grid;
  BArgs bb = b;
  bb.k.push_mode = get_push_mode();
  void* args[] = {&bb};
  const dim3 g3((unsigned)grid, (unsigned)grid_y), blk((unsigned)block);
  if (grid_y > 1) return cudaLaunchCooperativeKernel(fp, g3, blk, args, smem, stream);
  if (!get_dependent_launch()) return cudaLaunchKernel(fp, g3, blk, args, smem, stream);
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
  return cudaLaunchKernelExC(&cfg, fp, args);
}

cudaError_t launch_dw_reduce(const float* ws, int parts, int64_t hl, void* dw, int dtype,
                             cudaStream_t stream) {
  const dim3 grid((unsigned)((hl + 31) / 32)), blk(kDwWarps * 32);
  const void* fn = dtype == kF32    ? reinterpret_cast<const void*>(backward_dw_reduce_kernel<float>)
                   : dtype == kBF16 ? reinterpret_cast<const void*>(
                                          backward_dw_reduce_kernel<__nv_bfloat16>)
                                    : reinterpret_cast<const void*>(backward_dw_reduce_kernel<__half>);
  void* args[] = {&ws, &parts, &hl, &dw};
  if (!get_dependent_launch()) return cudaLaunchKernel(fn, grid, blk, args, 0, stream);
  // launched while the backward kernel drains; waits for it in griddepcontrol.wait
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = blk;
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelExC(&cfg, fn, args);
}

}  // namespace rtp
