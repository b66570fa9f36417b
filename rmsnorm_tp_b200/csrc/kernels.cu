// Fused tensor-parallel RMSNorm kernels for B200 (sm_100a).
//
// One launch per forward call. For each row r of x [rows, hl] on rank k:
//   1. load the row with 128-bit loads into registers (read once from HBM),
//   2. s_k = sum(x^2) in fp32 (warp butterfly, then across the team's warps),
//   3. push {s_k, tag} into slot [buf][k][r] of every peer's mailbox (one
//      relaxed system-scope 64-bit store per peer over NVLink),
//   4. poll slots [buf][q][r] of the local mailbox until each carries the tag
//      (bounded by the global timer),
//   5. S = s_0 + s_1 + ... + s_{tp-1} in rank order (bit-identical on every rank),
//      y = (x * rsqrt(S / hidden + eps)) * w in fp32 from the registers, one
//      rounding to the output type, 128-bit stores.
// Reference: csrc/rmsnorm_tp.cu:48-178 does the same five phases with one CTA
// per row, a second read of x for phase 5, a separate flag word per slot and an
// unbounded `>=` poll; the math contract (S / hidden, rsqrtf, x*inv*w) follows
// rmsnorm_tp.cu:156-170 and the AllReduce path bench_rmsnorm_tp.py:16-22.
//
// Rows map to "teams" of W warps. A team walks row tiles in a grid-stride loop
// over a grid of at most one resident wave, so all CTAs of every rank are
// resident together and the waits between GPUs always make progress.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdlib>

#include "device_common.cuh"
#include "internal.h"
#include "ptx.cuh"
#include "rtp_common.h"

namespace rtp {

// ---------------------------------------------------------------------------
// Register kernel: a team of kW warps holds kRows rows in registers between
// the load and the store (x is read from HBM once), kVec 16-byte vectors per
// lane and row. Column vector c of a row belongs to lane c % 32 of warp
// (c / 32) % kW, register j = c / (32 kW): each warp instruction touches 512
// contiguous bytes.
//
// Three-buffer software pipeline per team. Buffers rotate through the roles
//   A: tile t    -- partial pushed one step ago; poll the peers' partials, store y
//   B: tile t+s  -- loads issued one step ago; reduce, push the partial
//   C: tile t+2s -- loads issued now
// and one step runs C-load, B-reduce-push, A-poll-store. Each tile's HBM
// latency is covered by the rest of the step it was issued in, and each tile's
// NVLink round trip (push -> peer's push visible) by a full step of other work,
// so neither latency adds up tile after tile.
// ---------------------------------------------------------------------------
template <typename T, int kVec, int kW, int kRows, int kBlock, int kMinBlocks>
__global__ void __launch_bounds__(kBlock, kMinBlocks)
    tp_rmsnorm_vec_kernel(const __grid_constant__ KArgs a) {
  constexpr int kTeams = kBlock / 32 / kW;
  static_assert(kTeams >= 1 && kTeams <= 15, "team count must fit the named barriers");
  static_assert(kRows * kMaxTP <= 32, "one warp serves every (row, rank) pair of a tile");
  ptx::grid_dep_wait();
  ptx::grid_dep_launch_dependents();
  const unsigned long long t_start = a.prof ? ptx::globaltimer() : 0ull;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int team = warp / kW;
  const int wit = warp - team * kW;
  const int ri = a.emulated ? (int)blockIdx.y : 0;
  const int rank = a.emulated ? (int)blockIdx.y : a.rank;
  const RankPtrs& rp = a.rp[ri];
  const int64_t V = a.hl / Pack<T>::kE;
  // x and out may be the same memory (in place): no __restrict__ on either
  const uint4* xg = ptx::launder(reinterpret_cast<const uint4*>(rp.x));
  const uint4* __restrict__ wg = ptx::launder(reinterpret_cast<const uint4*>(rp.w));
  uint4* yg = reinterpret_cast<uint4*>(rp.out);
  const bool exchange = a.tp > 1;
  const int tp = a.tp;
  const int lr = exchange ? lane / tp : 0;      // exchange lane -> (row, rank)
  const int lq = exchange ? lane - lr * tp : 0;

  __shared__ float s_part[kTeams][3][kW][kRows];
  __shared__ float s_sum[kTeams][3][kRows];
  __shared__ int s_ok[kTeams][3];

  const int64_t tiles = (a.rows + kRows - 1) / kRows;
  const int64_t stride = (int64_t)gridDim.x * kTeams;
  int64_t t = (int64_t)blockIdx.x * kTeams + team;

  unsigned long long call = 0ull;
  uint32_t buf = 0u, tag = 0u;
  WaitStats ws;

  auto nrows_of = [&](int64_t tt) { return (int)min((int64_t)kRows, a.rows - tt * kRows); };
  // this thread's weight vectors -> L1 while the first loads are in flight, so
  // the normalisation's weight reads (after the reduction and the exchange)
  // hit L1 instead of waiting an L2 round trip
  auto prefetch_weights = [&] {
#pragma unroll
    for (int j = 0; j < kVec; ++j) {
      const int c = (j * kW + wit) * 32 + lane;
      if (c < V) ptx::prefetch_l1(wg + c);
    }
  };

  auto load = [&](int64_t tt, uint4 (&xv)[kRows][kVec]) {
    const int64_t row0 = tt * kRows;
    const int nr = nrows_of(tt);
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
      const uint4* xr = xg + (row0 + r) * V;
#pragma unroll
      for (int j = 0; j < kVec; ++j) {
        const int c = (j * kW + wit) * 32 + lane;
        if (r < nr && c < V)
          xv[r][j] = ptx::ld_stream_v4(xr + c);
        else
          xv[r][j] = make_uint4(0u, 0u, 0u, 0u);
      }
    }
  };

  // Team-wide fp32 sum of squares of each row (every lane of the team gets it).
  auto reduce = [&](const uint4 (&xv)[kRows][kVec], float (&ss)[kRows], int slot) {
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
      float s = 0.f;
#pragma unroll
      for (int j = 0; j < kVec; ++j) s += sumsq16<T>(xv[r][j]);
      ss[r] = warp_allreduce_sum(s);
    }
    if constexpr (kW > 1) {
      if (lane == 0) {
#pragma unroll
        for (int r = 0; r < kRows; ++r) s_part[team][slot][wit][r] = ss[r];
      }
      ptx::team_bar(1 + team, kW * 32);
#pragma unroll
      for (int r = 0; r < kRows; ++r) {
        float s = 0.f;
#pragma unroll
        for (int w = 0; w < kW; ++w) s += s_part[team][slot][w][r];
        ss[r] = s;
      }
    }
  };

  auto mine_of = [&](const float (&ss)[kRows]) {
    float m = 0.f;
#pragma unroll
    for (int i = 0; i < kRows; ++i)
      if (i == lr) m = ss[i];
    return m;
  };

  auto push = [&](int64_t tt, const float (&ss)[kRows]) {
    if (kW == 1 || wit == 0)
      push_slot(a, rank, buf, tag, tt * kRows + lr, lq, lr < nrows_of(tt), mine_of(ss));
  };

  // Group sums S of tile tt's rows (rank order); false if a wait gave up.
  auto gather = [&](int64_t tt, const float (&ss)[kRows], float (&S)[kRows], int slot) {
    bool ok = true;
    if (!exchange) {
#pragma unroll
      for (int r = 0; r < kRows; ++r) S[r] = ss[r];
      return ok;
    }
    if (kW == 1 || wit == 0) {
      bool failed = false;
      const float val = poll_slot(a, rank, rp, buf, tag, call, tt * kRows + lr, lq,
                                  lr < nrows_of(tt), mine_of(ss), failed, ws);
      ok = !__any_sync(0xFFFFFFFFu, failed);
#pragma unroll
      for (int i = 0; i < kRows; ++i) {
        float s = 0.f;
        for (int p = 0; p < tp; ++p) s += __shfl_sync(0xFFFFFFFFu, val, i * tp + p);
        S[i] = s;
      }
    }
    if constexpr (kW > 1) {
      if (wit == 0 && lane == 0) {
#pragma unroll
        for (int r = 0; r < kRows; ++r) s_sum[team][slot][r] = S[r];
        s_ok[team][slot] = ok ? 1 : 0;
      }
      ptx::team_bar(1 + team, kW * 32);
#pragma unroll
      for (int r = 0; r < kRows; ++r) S[r] = s_sum[team][slot][r];
      ok = s_ok[team][slot] != 0;
    }
    return ok;
  };

  auto store = [&](int64_t tt, const uint4 (&xv)[kRows][kVec], const float (&S)[kRows], bool ok) {
    const int64_t row0 = tt * kRows;
    const int nr = nrows_of(tt);
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
      if (r < nr) {
        const float inv = ok ? rsqrtf(S[r] / a.hidden_f + a.eps) : quiet_nan();
        uint4* yr = yg + (row0 + r) * V;
#pragma unroll
        for (int j = 0; j < kVec; ++j) {
          const int c = (j * kW + wit) * 32 + lane;
          if (c < V) ptx::st_v4(yr + c, normalize16<T>(xv[r][j], ptx::ld_cached_v4(wg + c), inv));
        }
      }
    }
  };

  // One step with buffer roles (A, B, C) = tiles (tt, tt + stride, tt + 2 stride);
  // returns false once tile tt was the team's last.
  auto step = [&](int64_t tt, uint4 (&xa)[kRows][kVec], float (&ssa)[kRows], int sa,
                  uint4 (&xb)[kRows][kVec], float (&ssb)[kRows], int sb,
                  uint4 (&xc)[kRows][kVec]) {
    const int64_t t1 = tt + stride, t2 = tt + 2 * stride;
    if (t2 < tiles) load(t2, xc);
    if (t1 < tiles) {
      reduce(xb, ssb, sb);
      if (exchange) push(t1, ssb);
    }
    float S[kRows];
    const bool ok = gather(tt, ssa, S, sa);
    store(tt, xa, S, ok);
    return t1 < tiles;
  };

  if (t < tiles) {
    uint4 x0[kRows][kVec], x1[kRows][kVec], x2[kRows][kVec];
    float ss0[kRows], ss1[kRows], ss2[kRows];
    load(t, x0);
    if (t + stride < tiles) load(t + stride, x1);
    prefetch_weights();
    if (exchange) {   // read after the first loads are in flight: its latency overlaps theirs
      call = read_generation(rp.state);
      buf = buffer_of(call);
      tag = tag_of(call);
    }
    reduce(x0, ss0, 0);
    if (exchange) push(t, ss0);
    for (;;) {
      if (!step(t, x0, ss0, 0, x1, ss1, 1, x2)) break;
      t += stride;
      if (!step(t, x1, ss1, 1, x2, ss2, 2, x0)) break;
      t += stride;
      if (!step(t, x2, ss2, 2, x0, ss0, 0, x1)) break;
      t += stride;
    }
  } else if (exchange) {
    call = read_generation(rp.state);
  }
  if (exchange) finish_launch(rp.state, call);
  flush_stats(a, ws, t_start);
}

// ---------------------------------------------------------------------------
// Resident register kernel (TP > 1, calls of at most kDepth tiles per team):
// the same teams, tiles, column mapping and exchange as the register kernel
// above, but every tile of a team is held in registers at once. All of a
// team's loads are issued first (every byte of the call is in flight at once),
// then each tile is reduced and its partials pushed as its data arrives, then
// each tile's peers' partials are polled and the tile normalised and stored.
// The NVLink round trip of a tile overlaps the loads and reductions of the
// team's later tiles instead of waiting behind a three-buffer rotation.
// ---------------------------------------------------------------------------
template <typename T, int kVec, int kW, int kRows, int kBlock, int kMinBlocks, int kDepth>
__global__ void __launch_bounds__(kBlock, kMinBlocks)
    tp_rmsnorm_vec_resident_kernel(const __grid_constant__ KArgs a) {
  constexpr int kTeams = kBlock / 32 / kW;
  static_assert(kTeams >= 1 && kTeams <= 15, "team count must fit the named barriers");
  static_assert(kRows * kMaxTP <= 32, "one warp serves every (row, rank) pair of a tile");
  ptx::grid_dep_wait();
  ptx::grid_dep_launch_dependents();
  const unsigned long long t_start = a.prof ? ptx::globaltimer() : 0ull;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int team = warp / kW;
  const int wit = warp - team * kW;
  const int ri = a.emulated ? (int)blockIdx.y : 0;
  const int rank = a.emulated ? (int)blockIdx.y : a.rank;
  const RankPtrs& rp = a.rp[ri];
  const int64_t V = a.hl / Pack<T>::kE;
  // x and out may be the same memory (in place): no __restrict__ on either
  const uint4* xg = ptx::launder(reinterpret_cast<const uint4*>(rp.x));
  const uint4* __restrict__ wg = ptx::launder(reinterpret_cast<const uint4*>(rp.w));
  uint4* yg = reinterpret_cast<uint4*>(rp.out);
  const int tp = a.tp;
  const int lr = lane / tp;      // exchange lane -> (row, rank)
  const int lq = lane - lr * tp;

  __shared__ float s_part[kTeams][kDepth][kW][kRows];
  __shared__ float s_sum[kTeams][kDepth][kRows];
  __shared__ int s_ok[kTeams][kDepth];
  __shared__ float s_cpart[kDepth][kTeams * kRows];   // the CTA's partials, per depth
  static_assert(kTeams * kRows <= 32, "one lane per row of a CTA's depth level");
  static_assert(kBlock / 32 >= kMaxTP, "one warp per peer");

  const int64_t tiles = (a.rows + kRows - 1) / kRows;
  const int64_t stride = (int64_t)gridDim.x * kTeams;
  const int64_t first = (int64_t)blockIdx.x * kTeams + team;
  WaitStats ws;
  auto nrows_of = [&](int64_t tt) { return (int)min((int64_t)kRows, a.rows - tt * kRows); };
  auto mine_of = [&](const float (&ss)[kRows]) {
    float m = 0.f;
#pragma unroll
    for (int i = 0; i < kRows; ++i)
      if (i == lr) m = ss[i];
    return m;
  };

  uint4 xv[kDepth][kRows][kVec];
  float ss[kDepth][kRows];
#pragma unroll
  for (int d = 0; d < kDepth; ++d) {
    const int64_t tt = first + d * stride;
    const int nr = tt < tiles ? nrows_of(tt) : 0;
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
      const uint4* xr = xg + (tt * kRows + r) * V;
#pragma unroll
      for (int j = 0; j < kVec; ++j) {
        const int c = (j * kW + wit) * 32 + lane;
        xv[d][r][j] = (r < nr && c < V) ? ptx::ld_stream_v4(xr + c) : make_uint4(0u, 0u, 0u, 0u);
      }
    }
  }
  // this thread's weight vectors -> L1 while the loads are in flight (the
  // normalisation reads them after the exchange)
#pragma unroll
  for (int j = 0; j < kVec; ++j) {
    const int c = (j * kW + wit) * 32 + lane;
    if (c < V && first < tiles) ptx::prefetch_l1(wg + c);
  }
  const unsigned long long call = read_generation(rp.state);
  const uint32_t buf = buffer_of(call), tag = tag_of(call);

  // Reduce every tile as its loads complete and push it. At depth d the CTA's
  // teams hold kTeams consecutive tiles = kTeams * kRows consecutive rows, so
  // after a CTA barrier warp q writes all of them to rank q as ONE contiguous
  // store of kTeams * kRows slots (one NVLink write per peer, CTA and depth,
  // instead of one per peer and team).
  const int64_t cta_tile0 = (int64_t)blockIdx.x * kTeams;
  const bool xlane = kW == 1 || wit == 0;   // the team's exchange warp
  auto reduce_push = [&](int d) {
    const int64_t tt = first + d * stride;
    if (tt < tiles) {
#pragma unroll
      for (int r = 0; r < kRows; ++r) {
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < kVec; ++j) s += sumsq16<T>(xv[d][r][j]);
        ss[d][r] = warp_allreduce_sum(s);
      }
      if constexpr (kW > 1) {
        if (lane == 0) {
#pragma unroll
          for (int r = 0; r < kRows; ++r) s_part[team][d][wit][r] = ss[d][r];
        }
        ptx::team_bar(1 + team, kW * 32);
#pragma unroll
        for (int r = 0; r < kRows; ++r) {
          float s = 0.f;
#pragma unroll
          for (int w = 0; w < kW; ++w) s += s_part[team][d][w][r];
          ss[d][r] = s;
        }
      }
      if (xlane && lane < kRows) {
        float m = 0.f;
#pragma unroll
        for (int r = 0; r < kRows; ++r)
          if (r == lane) m = ss[d][r];
        s_cpart[d][team * kRows + lane] = m;
      }
    }
    __syncthreads();
    if (warp < tp && warp != rank && lane < kTeams * kRows) {
      const int64_t row = (cta_tile0 + d * stride) * kRows + lane;
      if (row < a.rows)
        store_slot(a.push_mode, a.mbox[warp] + slot_index(buf, rank, tp, a.nmax, row),
                   s_cpart[d][lane], tag);
    }
  };
  // one look at a tile's slot (packed encoding; the release encoding's acquire
  // must precede its value read, so it polls in finish)
  auto probe = [&](int d) -> unsigned long long {
    const int64_t tt = first + d * stride;
    const bool remote = xlane && tt < tiles && lr < nrows_of(tt) && lq != rank;
    return remote && a.push_mode == kPushPacked
               ? ptx::ld_relaxed_sys_u64(a.mbox[rank] +
                                         slot_index(buf, lq, tp, a.nmax, tt * kRows + lr))
               : 0ull;
  };
  // the peers' partials of a tile (the probed word, else a bounded poll), the
  // team's sum, then normalise and store the tile from the registers
  auto finish = [&](int d, unsigned long long seen) {
    const int64_t tt = first + d * stride;
    if (tt >= tiles) return;   // uniform over the team
    float S[kRows];
    bool ok = true;
    if (xlane) {
      bool failed = false;
      const bool active = lr < nrows_of(tt);
      float val;
      if (!active || lq == rank) {
        val = mine_of(ss[d]);
      } else if (a.push_mode == kPushPacked && slot_tag(seen) == tag) {
        ws.fast += 1;
        val = slot_value(seen);
      } else {
        val = poll_slot(a, rank, rp, buf, tag, call, tt * kRows + lr, lq, true, 0.f, failed, ws);
      }
      ok = !__any_sync(0xFFFFFFFFu, failed);
#pragma unroll
      for (int i = 0; i < kRows; ++i) {
        float s = 0.f;
        for (int p = 0; p < tp; ++p) s += __shfl_sync(0xFFFFFFFFu, val, i * tp + p);
        S[i] = s;
      }
    }
    if constexpr (kW > 1) {
      if (wit == 0 && lane == 0) {
#pragma unroll
        for (int r = 0; r < kRows; ++r) s_sum[team][d][r] = S[r];
        s_ok[team][d] = ok ? 1 : 0;
      }
      ptx::team_bar(1 + team, kW * 32);
#pragma unroll
      for (int r = 0; r < kRows; ++r) S[r] = s_sum[team][d][r];
      ok = s_ok[team][d] != 0;
    }
    const int nr = nrows_of(tt);
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
      if (r < nr) {
        const float inv = ok ? rsqrtf(S[r] / a.hidden_f + a.eps) : quiet_nan();
        uint4* yr = yg + (tt * kRows + r) * V;
#pragma unroll
        for (int j = 0; j < kVec; ++j) {
          const int c = (j * kW + wit) * 32 + lane;
          if (c < V) ptx::st_v4(yr + c, normalize16<T>(xv[d][r][j], ptx::ld_cached_v4(wg + c), inv));
        }
      }
    }
  };

  // Depth f is finished kLag depths after its push, so its stores overlap the
  // loads and reductions of the later depths and its peers' partials have an
  // NVLink round trip's worth of that work to arrive; its slot is probed
  // before the reduction in between (the probe's round trip overlaps it).
  // Every push precedes every wait on a depth at least kLag lower, on every
  // rank, so the waits end.
  constexpr int kLag = kDepth > 2 ? 2 : kDepth - 1;
  unsigned long long seen[kDepth];
#pragma unroll
  for (int d = 0; d < kDepth; ++d) {
    if (d >= kLag) seen[d - kLag] = probe(d - kLag);
    if (cta_tile0 + d * stride < tiles) reduce_push(d);   // uniform over the CTA
    if (d >= kLag) finish(d - kLag, seen[d - kLag]);
  }
  const unsigned long long t_mid = a.prof ? ptx::globaltimer() : 0ull;
#pragma unroll
  for (int d = kDepth - kLag; d < kDepth; ++d) seen[d] = probe(d);
#pragma unroll
  for (int d = kDepth - kLag; d < kDepth; ++d) finish(d, seen[d]);
  finish_launch(rp.state, call);
  flush_stats(a, ws, t_start, t_mid);
}

// ---------------------------------------------------------------------------
// Local register kernel (TP = 1, no exchange). Same teams, tiles and column
// mapping as the register kernel above, but without the exchange there is no
// tile waiting for peers, so every buffer holds loads in flight: a team keeps
// kDepth tiles in flight, reduces and stores its oldest straight from the
// registers and refills that buffer with the tile kDepth strides ahead.
// kRes: fused residual add -- each buffer also holds the residual rows;
// z = x + r (rounded to T) is written back to the residual and normalised.
// ---------------------------------------------------------------------------
template <typename T, int kVec, int kW, int kRows, int kBlock, int kMinBlocks, int kDepth,
          bool kRes = false>
__global__ void __launch_bounds__(kBlock, kMinBlocks)
    rmsnorm_local_vec_kernel(const __grid_constant__ KArgs a) {
  constexpr int kTeams = kBlock / 32 / kW;
  static_assert(kTeams >= 1 && kTeams <= 15, "team count must fit the named barriers");
  static_assert(kDepth >= 2, "at least two tiles in flight");
  ptx::grid_dep_wait();
  ptx::grid_dep_launch_dependents();
  const unsigned long long t_start = a.prof ? ptx::globaltimer() : 0ull;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int team = warp / kW;
  const int wit = warp - team * kW;
  const RankPtrs& rp = a.rp[0];
  const int64_t V = a.hl / Pack<T>::kE;
  // x and out may be the same memory (in place), and the residual is read and
  // rewritten: no __restrict__ on any of them
  const uint4* xg = ptx::launder(reinterpret_cast<const uint4*>(rp.x));
  const uint4* __restrict__ wg = ptx::launder(reinterpret_cast<const uint4*>(rp.w));
  uint4* yg = reinterpret_cast<uint4*>(rp.out);
  uint4* rg = kRes ? ptx::launder(reinterpret_cast<uint4*>(rp.res)) : nullptr;

  // two slots: a warp rewrites slot s only after the next team barrier, which
  // every warp of the team reaches after reading slot s
  __shared__ float s_part[kTeams][2][kW][kRows];

  const int64_t tiles = (a.rows + kRows - 1) / kRows;
  const int64_t stride = (int64_t)gridDim.x * kTeams;
  const int64_t first = (int64_t)blockIdx.x * kTeams + team;

  auto nrows_of = [&](int64_t tt) { return (int)min((int64_t)kRows, a.rows - tt * kRows); };

  auto load = [&](int64_t tt, uint4 (&xv)[kRows][kVec], uint4 (&rv)[kRows][kVec]) {
    const int64_t row0 = tt * kRows;
    const int nr = nrows_of(tt);
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
      const uint4* xr = xg + (row0 + r) * V;
#pragma unroll
      for (int j = 0; j < kVec; ++j) {
        const int c = (j * kW + wit) * 32 + lane;
        if (r < nr && c < V) {
          xv[r][j] = ptx::ld_stream_v4(xr + c);
          if constexpr (kRes) rv[r][j] = ptx::ld_stream_v4(rg + (row0 + r) * V + c);
        } else {
          xv[r][j] = make_uint4(0u, 0u, 0u, 0u);
          if constexpr (kRes) rv[r][j] = make_uint4(0u, 0u, 0u, 0u);
        }
      }
    }
  };

  // (kRes: z = x + r into xv, written back to the residual) team-wide fp32 sum
  // of squares, then y from the registers
  auto finish = [&](int64_t tt, uint4 (&xv)[kRows][kVec], const uint4 (&rv)[kRows][kVec],
                    int slot) {
    if constexpr (kRes) {
      const int64_t row0 = tt * kRows;
      const int nr = nrows_of(tt);
#pragma unroll
      for (int r = 0; r < kRows; ++r) {
#pragma unroll
        for (int j = 0; j < kVec; ++j) {
          const int c = (j * kW + wit) * 32 + lane;
          xv[r][j] = add16<T>(xv[r][j], rv[r][j]);
          if (r < nr && c < V) ptx::st_v4(rg + (row0 + r) * V + c, xv[r][j]);
        }
      }
    }
    float ss[kRows];
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
      float s = 0.f;
#pragma unroll
      for (int j = 0; j < kVec; ++j) s += sumsq16<T>(xv[r][j]);
      ss[r] = warp_allreduce_sum(s);
    }
    if constexpr (kW > 1) {
      if (lane == 0) {
#pragma unroll
        for (int r = 0; r < kRows; ++r) s_part[team][slot][wit][r] = ss[r];
      }
      ptx::team_bar(1 + team, kW * 32);
#pragma unroll
      for (int r = 0; r < kRows; ++r) {
        float s = 0.f;
#pragma unroll
        for (int w = 0; w < kW; ++w) s += s_part[team][slot][w][r];
        ss[r] = s;
      }
    }
    const int64_t row0 = tt * kRows;
    const int nr = nrows_of(tt);
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
      if (r < nr) {
        const float inv = rsqrtf(ss[r] / a.hidden_f + a.eps);
        uint4* yr = yg + (row0 + r) * V;
#pragma unroll
        for (int j = 0; j < kVec; ++j) {
          const int c = (j * kW + wit) * 32 + lane;
          if (c < V) ptx::st_v4(yr + c, normalize16<T>(xv[r][j], ptx::ld_cached_v4(wg + c), inv));
        }
      }
    }
  };

  uint4 xb[kDepth][kRows][kVec];
  uint4 rb[kRes ? kDepth : 1][kRows][kVec];   // residual rows (kRes only)
#pragma unroll
  for (int d = 0; d < kDepth; ++d)
    if (first + d * stride < tiles) load(first + d * stride, xb[d], rb[kRes ? d : 0]);
  // this thread's weight vectors -> L1 while the first loads are in flight
#pragma unroll
  for (int j = 0; j < kVec; ++j) {
    const int c = (j * kW + wit) * 32 + lane;
    if (c < V && first < tiles) ptx::prefetch_l1(wg + c);
  }
  int slot = 0;
  for (int64_t base = first; base < tiles; base += kDepth * stride) {
#pragma unroll
    for (int d = 0; d < kDepth; ++d) {
      const int64_t tt = base + d * stride;
      if (tt >= tiles) break;
      finish(tt, xb[d], rb[kRes ? d : 0], slot);
      slot ^= 1;
      if (tt + kDepth * stride < tiles) load(tt + kDepth * stride, xb[d], rb[kRes ? d : 0]);
    }
  }
  flush_stats(a, WaitStats{}, t_start);
}

// ---------------------------------------------------------------------------
// Generic kernel: any width and alignment. One CTA per row at a time, scalar
// loads, x read twice (the second read normally hits L2). Same exchange.
// ---------------------------------------------------------------------------
template <typename T, int kBlock, bool kRes = false>
__global__ void __launch_bounds__(kBlock)
    tp_rmsnorm_generic_kernel(const __grid_constant__ KArgs a) {
  constexpr int kWarps = kBlock / 32;
  ptx::grid_dep_wait();
  ptx::grid_dep_launch_dependents();
  const unsigned long long t_start = a.prof ? ptx::globaltimer() : 0ull;
  WaitStats ws;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int ri = a.emulated ? (int)blockIdx.y : 0;
  const int rank = a.emulated ? (int)blockIdx.y : a.rank;
  const RankPtrs& rp = a.rp[ri];
  const T* xg = reinterpret_cast<const T*>(rp.x);    // may be out (in place)
  const T* __restrict__ wg = reinterpret_cast<const T*>(rp.w);
  T* yg = reinterpret_cast<T*>(rp.out);
  T* rg = reinterpret_cast<T*>(rp.res);   // kRes: residual, rewritten with z = x + r
  const bool exchange = a.tp > 1;
  const int64_t hl = a.hl;

  __shared__ unsigned long long s_call;
  __shared__ float s_part[kWarps];
  __shared__ float s_sum;
  __shared__ int s_ok;

  unsigned long long call = 0ull;
  uint32_t buf = 0u, tag = 0u;
  if (exchange) {
    if (threadIdx.x == 0) s_call = read_generation(rp.state);
    __syncthreads();
    call = s_call;
    buf = buffer_of(call);
    tag = tag_of(call);
  }

  for (int64_t row = blockIdx.x; row < a.rows; row += gridDim.x) {
    const T* xr = xg + row * hl;
    float s = 0.f;
    for (int64_t i = threadIdx.x; i < hl; i += kBlock) {
      float v = Pack<T>::to_f(xr[i]);
      if constexpr (kRes) {
        const T z = Pack<T>::from_f(v + Pack<T>::to_f(rg[row * hl + i]));
        rg[row * hl + i] = z;
        v = Pack<T>::to_f(z);
      }
      s = fmaf(v, v, s);
    }
    s = warp_allreduce_sum(s);
    if (lane == 0) s_part[warp] = s;
    __syncthreads();
    if (warp == 0) {
      float t = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) t += s_part[w];
      float ss[1] = {t};
      float S[1] = {t};
      bool ok = true;
      if (exchange) {
        bool failed = false;
        const int q = lane;   // tp <= 8 lanes serve the row's ranks
        const float val = push_poll(a, rank, rp, buf, tag, call, row, q, q < a.tp, ss[0], failed, ws);
        ok = !__any_sync(0xFFFFFFFFu, failed);
        float tot = 0.f;
        for (int p = 0; p < a.tp; ++p) tot += __shfl_sync(0xFFFFFFFFu, val, p);
        S[0] = tot;
      }
      if (lane == 0) {
        s_sum = S[0];
        s_ok = ok ? 1 : 0;
      }
    }
    __syncthreads();
    const float var = s_sum / a.hidden_f;
    const float inv = s_ok ? rsqrtf(var + a.eps) : quiet_nan();
    T* yr = yg + row * hl;
    const T* zr = kRes ? rg + row * hl : xr;   // this thread's own residual writes above
    for (int64_t i = threadIdx.x; i < hl; i += kBlock) {
      const float v = Pack<T>::to_f(zr[i]);
      const float w = Pack<T>::to_f(wg[i]);
      yr[i] = Pack<T>::from_f((v * inv) * w);
    }
    __syncthreads();  // s_part / s_sum are reused by the next row
  }
  if (exchange) finish_launch(rp.state, call);
  flush_stats(a, ws, t_start);
}

// ---------------------------------------------------------------------------
// Bulk-copy kernel (the default for aligned rows of up to 16 KB).
//
// Every warp owns a ring of kStages shared-memory stages. A stage holds one
// tile of tile_rows consecutive rows -- one contiguous span of x -- fetched by a
// single cp.async.bulk (TMA) copy that signals an mbarrier with its byte
// count, so the bytes in flight per SM are set by shared memory (~200 KB),
// not by registers. The weight row is staged once per CTA. x is read from HBM
// once (then from shared memory for the sum of squares and the normalisation);
// y is written with 128-bit stores.
//
// Per warp, tile k goes through: wait for its copy -> reduce -> push the
// partials -> [lag] -> poll the peers' partials -> normalise, store -> refill
// its stage with tile k + kStages. The poll of tile k waits until `lag` more
// tiles have been reduced and pushed, so the NVLink round trip -- and the
// progress skew between ranks, which grows with the number of peers --
// overlaps that much work; each copy is issued kStages - lag - 1 tiles before
// it is needed. (A lag of one tile is kept at TP = 1 too, where it measured
// faster than none.) Tiles go to warps round-robin (tile t -> warp
// t mod all warps), the same on every rank, over at most one resident wave.
// ---------------------------------------------------------------------------

// kRes (fused residual add): a stage holds the x tile and, stage_bytes / 2
// further, the residual tile (two copies on the same mbarrier); the reduction
// writes z = x + r (rounded to T) over the x tile and to the residual in HBM,
// and the normalisation reads z.
template <typename T, int kWarps, int kStages, int kRowsMax, bool kRes = false>
__global__ void __launch_bounds__(kWarps * 32, 1)
    tp_rmsnorm_bulk_kernel(const __grid_constant__ KArgs a) {
  static_assert(kRowsMax >= 1 && kRowsMax <= 32, "rows per tile");
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ __align__(8) unsigned long long s_bar[kWarps][kStages];
  __shared__ float s_part[kWarps][kStages][32];   // partials of the tile in each stage
  __shared__ float s_sum[kWarps][32];
  __shared__ unsigned long long s_call;

  ptx::grid_dep_wait();
  ptx::grid_dep_launch_dependents();
  const unsigned long long t_start = a.prof ? ptx::globaltimer() : 0ull;
  WaitStats ws;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int ri = a.emulated ? (int)blockIdx.y : 0;
  const int rank = a.emulated ? (int)blockIdx.y : a.rank;
  const RankPtrs& rp = a.rp[ri];
  // tiles reduced (and pushed) but not yet finished: up to `lag`; copies are
  // issued kStages - lag - 1 tiles ahead of use
  const int lag = a.lag < 1 ? 1 : (a.lag > kStages - 2 ? kStages - 2 : a.lag);
  const int V = (int)(a.hl / Pack<T>::kE);                  // 16-byte vectors per row
  const uint32_t row_bytes = (uint32_t)a.hl * (uint32_t)sizeof(T);
  const uint32_t w_bytes = (row_bytes + 127u) & ~127u;
  const int tile_rows = a.tile_rows;
  const uint32_t stage_bytes = a.stage_bytes;
  const bool exchange = a.tp > 1;
  const int tp = a.tp;
  const int lr = exchange ? lane / tp : 0;      // exchange lane -> (row, rank)
  const int lq = exchange ? lane - lr * tp : 0;

  unsigned char* ring = smem + w_bytes + (size_t)warp * kStages * stage_bytes;
  const uint32_t ring_addr = ptx::smem_addr(ring);
  const uint32_t bar0 = ptx::smem_addr(&s_bar[warp][0]);
  const int64_t tiles = (a.rows + tile_rows - 1) / tile_rows;
  const int64_t nw = (int64_t)gridDim.x * kWarps;
  const int64_t wgid = (int64_t)blockIdx.x * kWarps + warp;
  const int64_t my_tiles = wgid < tiles ? (tiles - 1 - wgid) / nw + 1 : 0;
  const unsigned char* xg = reinterpret_cast<const unsigned char*>(rp.x);
  unsigned char* rg = reinterpret_cast<unsigned char*>(rp.res);   // kRes only
  const uint32_t res_off = kRes ? stage_bytes / 2u : 0u;          // residual tile in a stage

  auto row0_of = [&](int64_t kk) { return (wgid + kk * nw) * tile_rows; };
  auto nrows_of = [&](int64_t kk) { return (int)min((int64_t)tile_rows, a.rows - row0_of(kk)); };

  auto issue = [&](int64_t kk) {   // lane 0: fetch the warp's kk-th tile into stage kk % kStages
    const int st = (int)(kk % kStages);
    const uint32_t bytes = (uint32_t)nrows_of(kk) * row_bytes;
    const uint32_t bar = bar0 + 8u * (uint32_t)st;
    ptx::mbar_arrive_expect_tx(bar, kRes ? 2u * bytes : bytes);
    ptx::bulk_load(ring_addr + (uint32_t)st * stage_bytes, xg + row0_of(kk) * (int64_t)row_bytes,
                   bytes, bar);
    if constexpr (kRes)
      ptx::bulk_load(ring_addr + (uint32_t)st * stage_bytes + res_off,
                     rg + row0_of(kk) * (int64_t)row_bytes, bytes, bar);
  };

  int64_t issued = my_tiles < kStages ? my_tiles : kStages;
  if (lane == 0) {
#pragma unroll
    for (int st = 0; st < kStages; ++st) ptx::mbar_init(bar0 + 8u * st, 1u);
    ptx::fence_mbar_init();
    for (int64_t kk = 0; kk < issued; ++kk) issue(kk);
  }
  // weight row -> shared memory while the first tiles are in flight
  const uint4* wg = ptx::launder(reinterpret_cast<const uint4*>(rp.w));
  uint4* wsm = reinterpret_cast<uint4*>(smem);
  for (int v = threadIdx.x; v < V; v += kWarps * 32) wsm[v] = ptx::ld_cached_v4(wg + v);
  if (exchange && threadIdx.x == 0) s_call = read_generation(rp.state);
  __syncthreads();

  unsigned long long call = 0ull;
  uint32_t buf = 0u, tag = 0u;
  if (exchange) {
    call = s_call;
    buf = buffer_of(call);
    tag = tag_of(call);
  }
  uint4* yg = reinterpret_cast<uint4*>(rp.out);
  auto stage_ptr = [&](int64_t kk) {
    return reinterpret_cast<const uint4*>(ring + (size_t)(kk % kStages) * stage_bytes);
  };

  // sum of squares of every row of tile kk -> s_part[warp][kk % kStages][r]
  auto reduce = [&](int64_t kk) {
    const uint4* xs = stage_ptr(kk);
    const int nr = nrows_of(kk);
    if constexpr (kRes) {
      // z = x + r over the x tile and into the residual rows, then sum z^2
      uint4* zs = const_cast<uint4*>(xs);
      const uint4* rs = reinterpret_cast<const uint4*>(reinterpret_cast<const unsigned char*>(xs) +
                                                       res_off);
      uint4* rgt = reinterpret_cast<uint4*>(rg) + row0_of(kk) * (int64_t)V;
      for (int r = 0; r < nr; ++r) {
        float acc = 0.f;
        for (int v = lane; v < V; v += 32) {
          const uint4 z = add16<T>(zs[r * V + v], rs[r * V + v]);
          zs[r * V + v] = z;
          ptx::st_v4(rgt + r * V + v, z);
          acc += sumsq16<T>(z);
        }
        const float ss = warp_allreduce_sum(acc);
        if (lane == 0) s_part[warp][kk % kStages][r] = ss;
      }
    } else if (kRowsMax == 1 || (a.schedule & 1)) {
      for (int r = 0; r < nr; ++r) {
        const uint4* xr = xs + r * V;
        float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
        int v = lane;
        for (; v + 96 < V; v += 128) {
          a0 += sumsq16<T>(xr[v]);
          a1 += sumsq16<T>(xr[v + 32]);
          a2 += sumsq16<T>(xr[v + 64]);
          a3 += sumsq16<T>(xr[v + 96]);
        }
        for (; v < V; v += 32) a0 += sumsq16<T>(xr[v]);
        const float ss = warp_allreduce_sum((a0 + a1) + (a2 + a3));
        if (lane == 0) s_part[warp][kk % kStages][r] = ss;
      }
    } else {
      // every iteration loads one vector of each row (independent loads), and
      // the rows' butterflies run interleaved (independent shuffle chains)
      float acc[kRowsMax];
#pragma unroll
      for (int r = 0; r < kRowsMax; ++r) acc[r] = 0.f;
      for (int v = lane; v < V; v += 32) {
#pragma unroll
        for (int r = 0; r < kRowsMax; ++r)
          if (r < nr) acc[r] += sumsq16<T>(xs[r * V + v]);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
        for (int r = 0; r < kRowsMax; ++r) acc[r] += __shfl_xor_sync(0xFFFFFFFFu, acc[r], o);
      }
      if (lane == 0) {
#pragma unroll
        for (int r = 0; r < kRowsMax; ++r)
          if (r < nr) s_part[warp][kk % kStages][r] = acc[r];
      }
    }
    __syncwarp();
  };

  auto push = [&](int64_t kk) {
    const bool active = lr < nrows_of(kk);
    push_slot(a, rank, buf, tag, row0_of(kk) + lr, lq, active,
              active ? s_part[warp][kk % kStages][lr] : 0.f);
  };

  // poll tile kk's remote partials, normalise and store it, refill its stage
  // the slot word of the next tile to finish, loaded one reduction ahead of its
  // use (packed encoding), so that its round trip overlaps that reduction
  unsigned long long pre_word = 0ull;
  int64_t pre_tile = -1;
  auto prefetch = [&](int64_t kk) {
    pre_tile = kk;
    const bool remote = lr < nrows_of(kk) && lq != rank && a.push_mode == kPushPacked;
    pre_word = remote ? ptx::ld_relaxed_sys_u64(a.mbox[rank] +
                                                slot_index(buf, lq, tp, a.nmax, row0_of(kk) + lr))
                      : 0ull;
  };

  auto finish = [&](int64_t kk) {
    const int64_t row0 = row0_of(kk);
    const int nr = nrows_of(kk);
    bool ok = true;
    if (exchange) {
      const bool active = lr < nr;
      bool failed = false;
      float val;
      if (active && lq != rank && pre_tile == kk && a.push_mode == kPushPacked &&
          slot_tag(pre_word) == tag) {
        ws.fast += 1;
        val = slot_value(pre_word);
      } else {
        val = poll_slot(a, rank, rp, buf, tag, call, row0 + lr, lq, active,
                        active ? s_part[warp][kk % kStages][lr] : 0.f, failed, ws);
      }
      ok = !__any_sync(0xFFFFFFFFu, failed);
      float S = 0.f;
      for (int p = 0; p < tp; ++p) S += __shfl_sync(0xFFFFFFFFu, val, lr * tp + p);
      if (active && lq == 0) s_sum[warp][lr] = S;
    } else if (lane < nr) {
      s_sum[warp][lane] = s_part[warp][kk % kStages][lane];
    }
    __syncwarp();
    const uint4* xs = stage_ptr(kk);
    float inv[kRowsMax];
#pragma unroll
    for (int r = 0; r < kRowsMax; ++r)
      inv[r] = (r < nr && ok) ? rsqrtf(s_sum[warp][r] / a.hidden_f + a.eps) : quiet_nan();
    if (kRowsMax == 1 || (a.schedule & 2)) {
#pragma unroll
      for (int r = 0; r < kRowsMax; ++r) {
        if (r < nr) {
          const uint4* xr = xs + r * V;
          uint4* yr = yg + (row0 + r) * (int64_t)V;
#pragma unroll 4
          for (int v = lane; v < V; v += 32) ptx::st_v4(yr + v, normalize16<T>(xr[v], wsm[v], inv[r]));
        }
      }
    } else {
      uint4* yt = yg + row0 * (int64_t)V;
      for (int v = lane; v < V; v += 32) {
        const uint4 wv = wsm[v];   // one weight load serves every row of the tile
#pragma unroll
        for (int r = 0; r < kRowsMax; ++r)
          if (r < nr) ptx::st_v4(yt + r * V + v, normalize16<T>(xs[r * V + v], wv, inv[r]));
      }
    }
    __syncwarp();
    if (lane == 0 && kk + kStages < my_tiles) {
      ptx::fence_proxy_async_smem();   // our reads of the stage before the copy that refills it
      issue(kk + kStages);
    }
    if (kk + kStages < my_tiles && kk + kStages + 1 > issued) issued = kk + kStages + 1;
  };

  int64_t k = 0;
  int64_t f = 0;                 // oldest tile not finished yet; tiles [f, k) are pending
  bool load_ok = true;
  for (; k < my_tiles; ++k) {
    if (!mbar_wait_bounded(bar0 + 8u * (uint32_t)(k % kStages), (uint32_t)((k / kStages) & 1),
                           kLoadTimeoutNs)) {
      load_ok = false;
      break;
    }
    if (exchange && k + 1 - f > lag) prefetch(f);   // f is finished in this iteration
    reduce(k);
    if (exchange) push(k);
    // finish tiles only `lag` tiles behind: their NVLink round trips (TP > 1)
    // and the next copies overlap the reductions in between
    while (k + 1 - f > lag) finish(f++);
  }
  if (load_ok)
    while (f < my_tiles) finish(f++);
  if (!load_ok) {
    // A copy never landed: record it, then wait (bounded) for the copies still
    // in flight so none of them lands in shared memory this CTA no longer owns.
    if (lane == 0 && rp.state != nullptr) {
      if (atomicCAS(&rp.state->err_code, 0u, (unsigned)kStatusLoadTimeout) == 0u) {
        rp.state->err_call = call;
        if (rp.host_flag != nullptr) {
          *reinterpret_cast<volatile unsigned int*>(rp.host_flag) = (unsigned)kStatusLoadTimeout;
          __threadfence_system();
        }
      }
      atomicExch(&rp.state->abort, 1u);
    }
    for (int64_t kk = k; kk < issued; ++kk)
      mbar_wait_bounded(bar0 + 8u * (uint32_t)(kk % kStages), (uint32_t)((kk / kStages) & 1),
                        kLoadTimeoutNs);
  }
  if (exchange) finish_launch(rp.state, call);
  flush_stats(a, ws, t_start);
}

// ---------------------------------------------------------------------------
// Batch kernel (TP > 1 default for aligned rows of up to 16 KB).
//
// Every CTA owns one contiguous block of rows, split into batches of
// tile_rows (<= 32) consecutive rows. A batch is one contiguous span of x,
// fetched by one cp.async.bulk into a ring of `depth` shared-memory slots; a
// CTA whose block fits its ring has every byte of it in flight from the start.
// Per batch, all warps:
//   reduce  -- the sum of squares of each row (one or several warps per row),
//   push    -- warp q writes the batch's partials into peer q's mailbox: lane j
//              stores row j's {partial, tag}, so one store instruction moves
//              the whole batch to that peer as one contiguous write of
//              tile_rows x 8 bytes (one NVLink write per peer and batch, instead
//              of one per peer and row),
// and `lag` batches later
//   poll    -- warp q reads rank q's slots of that batch from the local mailbox
//              (lanes = rows, one contiguous load per peer), bounded waits,
//   finish  -- S = s_0 + ... + s_{tp-1} in rank order, y = (x * rsqrt(S / H +
//              eps)) * w from shared memory, 128-bit stores; the slot is refilled.
// The lag lets each batch's NVLink round trip and the ranks' skew overlap the
// reduction of the next batches while the ring keeps HBM busy. Every rank maps
// rows to CTAs and batches the same way, pushes batch b before it polls batch
// b - lag (lag >= 1), and every CTA is resident (one wave), so every wait is
// for a push that precedes the waiter's own earlier-batch waits on the peer:
// the waits always end.
// ---------------------------------------------------------------------------
constexpr int kBatchMaxRows = 32;
constexpr int kBatchMaxSlots = 8;

template <typename T, int kWarps>
__global__ void __launch_bounds__(kWarps * 32, 16 / kWarps)
    tp_rmsnorm_batch_kernel(const __grid_constant__ KArgs a) {
  static_assert(kWarps >= kMaxTP, "one warp per rank in the exchange");
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ __align__(8) unsigned long long s_bar[kBatchMaxSlots];
  __shared__ float s_red[kBatchMaxRows][kWarps];         // per (row, warp part) sums
  __shared__ float s_part[kBatchMaxSlots][kBatchMaxRows];  // this rank's partials, by slot
  __shared__ float s_val[kMaxTP][kBatchMaxRows];           // every rank's partials of the batch
  __shared__ unsigned long long s_call;                    //   being finished
  __shared__ int s_fail;

  ptx::grid_dep_wait();
  ptx::grid_dep_launch_dependents();
  const unsigned long long t_start = a.prof ? ptx::globaltimer() : 0ull;
  WaitStats ws;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int ri = a.emulated ? (int)blockIdx.y : 0;
  const int rank = a.emulated ? (int)blockIdx.y : a.rank;
  const RankPtrs& rp = a.rp[ri];
  const bool exchange = a.tp > 1;
  const int tp = a.tp;
  const int V = (int)(a.hl / Pack<T>::kE);                   // 16-byte vectors per row
  const uint32_t row_bytes = (uint32_t)a.hl * (uint32_t)sizeof(T);
  const uint32_t w_bytes = (row_bytes + 127u) & ~127u;
  const int bR = a.tile_rows;
  const int nslots = a.depth;
  const uint32_t slot_bytes = a.stage_bytes;
  // warps per row (g, a power of two) and the rows one pass of the CTA covers
  const int g = bR >= kWarps ? 1 : kWarps / bR;
  const int rows_per_pass = kWarps / g;
  const int wrow = warp / g, wpart = warp - wrow * g;

  const int64_t batches = (a.rows + bR - 1) / bR;
  const int64_t b_lo = batches * (int64_t)blockIdx.x / (int64_t)gridDim.x;
  const int64_t b_hi = batches * ((int64_t)blockIdx.x + 1) / (int64_t)gridDim.x;
  const int64_t nb = b_hi - b_lo;
  // lag: batches pushed but not finished; with refills it leaves copies issued
  // at least two batches ahead of use
  int lag = a.lag < 1 ? 1 : a.lag;
  if (nb > nslots && lag > nslots - 3) lag = nslots - 3 < 1 ? 1 : nslots - 3;

  const unsigned char* xg = reinterpret_cast<const unsigned char*>(rp.x);
  uint4* yg = reinterpret_cast<uint4*>(rp.out);
  unsigned char* ring = smem + w_bytes;
  const uint32_t ring_addr = ptx::smem_addr(ring);
  const uint32_t bar0 = ptx::smem_addr(&s_bar[0]);
  auto row0_of = [&](int64_t kk) { return (b_lo + kk) * bR; };
  auto nrows_of = [&](int64_t kk) { return (int)min((int64_t)bR, a.rows - row0_of(kk)); };
  auto issue = [&](int64_t kk) {   // thread 0: batch kk -> slot kk % nslots
    const int st = (int)(kk % nslots);
    const uint32_t bytes = (uint32_t)nrows_of(kk) * row_bytes;
    const uint32_t bar = bar0 + 8u * (uint32_t)st;
    ptx::mbar_arrive_expect_tx(bar, bytes);
    ptx::bulk_load(ring_addr + (uint32_t)st * slot_bytes, xg + row0_of(kk) * (int64_t)row_bytes,
                   bytes, bar);
  };
  int64_t issued = 0;   // thread 0 only
  if (threadIdx.x == 0) {
    for (int st = 0; st < nslots; ++st) ptx::mbar_init(bar0 + 8u * st, 1u);
    ptx::fence_mbar_init();
    issued = nb < nslots ? nb : nslots;
    for (int64_t kk = 0; kk < issued; ++kk) issue(kk);
    if (exchange) s_call = read_generation(rp.state);
  }
  // weight row -> shared memory while the first batches are in flight
  const uint4* wg = ptx::launder(reinterpret_cast<const uint4*>(rp.w));
  uint4* wsm = reinterpret_cast<uint4*>(smem);
  for (int v = threadIdx.x; v < V; v += kWarps * 32) wsm[v] = ptx::ld_cached_v4(wg + v);
  __syncthreads();
  unsigned long long call = 0ull;
  uint32_t buf = 0u, tag = 0u;
  if (exchange) {
    call = s_call;
    buf = buffer_of(call);
    tag = tag_of(call);
  }
  auto slot_ptr = [&](int64_t kk) {
    return reinterpret_cast<const uint4*>(ring + (size_t)(kk % nslots) * slot_bytes);
  };

  bool load_ok = true;
  int64_t b = 0;
  for (; b < nb + lag; ++b) {
    // A: batch b has landed (every thread observes its barrier, bounded), and the
    // previous iteration's reads of the slot finished there are complete
    bool ok = true;
    if (b < nb)
      ok = mbar_wait_bounded(bar0 + 8u * (uint32_t)(b % nslots), (uint32_t)((b / nslots) & 1),
                             kLoadTimeoutNs);
    if (!__syncthreads_and(ok)) {
      load_ok = false;
      break;
    }
    const int64_t f = b - lag;   // batch finished in this iteration
    if (threadIdx.x == 0) {
      // every thread has finished batch f - 1 (read its slot and s_fail) before A;
      // this iteration's polls set s_fail only after barrier B
      s_fail = 0;
      if (f >= 1 && f - 1 + nslots < nb) {
        ptx::fence_proxy_async_smem();   // the reads of slot (f - 1) before its refill
        issue(f - 1 + nslots);
        issued = f + nslots;
      }
    }
    int nr = 0;
    if (b < nb) {   // reduce
      nr = nrows_of(b);
      const uint4* xs = slot_ptr(b);
      for (int r = wrow; r < nr; r += rows_per_pass) {
        const uint4* xr = xs + r * V;
        float a0 = 0.f, a1 = 0.f;
        int v = wpart * 32 + lane;
        for (; v + g * 32 < V; v += 2 * g * 32) {
          a0 += sumsq16<T>(xr[v]);
          a1 += sumsq16<T>(xr[v + g * 32]);
        }
        if (v < V) a0 += sumsq16<T>(xr[v]);
        const float s = warp_allreduce_sum(a0 + a1);
        if (lane == 0) s_red[r][wpart] = s;
      }
    }
    __syncthreads();   // B
    if (b < nb && warp < tp && lane < nr) {   // push batch b: warp q -> rank q
      float part = 0.f;
      for (int k = 0; k < g; ++k) part += s_red[lane][k];
      if (warp == rank) {
        s_part[b % nslots][lane] = part;
      } else {
        unsigned long long* dst =
            a.mbox[warp] + slot_index(buf, rank, tp, a.nmax, row0_of(b) + lane);
        store_slot(a.push_mode, dst, part, tag);
      }
    }
    if (f >= 0 && warp < tp) {   // poll batch f: warp q <- rank q (lanes = rows)
      const int nrf = nrows_of(f);
      const bool active = lane < nrf;
      bool failed = false;
      const float mine = active && warp == rank ? s_part[f % nslots][lane] : 0.f;
      const float val = poll_slot(a, rank, rp, buf, tag, call, row0_of(f) + lane, warp, active,
                                  mine, failed, ws);
      if (active) s_val[warp][lane] = val;
      if (failed) s_fail = 1;
    }
    __syncthreads();   // C
    if (f >= 0) {      // finish batch f
      const int nrf = nrows_of(f);
      const uint4* xs = slot_ptr(f);
      const bool bad = s_fail != 0;
      for (int r = wrow; r < nrf; r += rows_per_pass) {
        float S = 0.f;
        for (int q = 0; q < tp; ++q) S += s_val[q][r];
        const float inv = bad ? quiet_nan() : rsqrtf(S / a.hidden_f + a.eps);
        const uint4* xr = xs + r * V;
        uint4* yr = yg + (row0_of(f) + r) * (int64_t)V;
#pragma unroll 2
        for (int v = wpart * 32 + lane; v < V; v += g * 32)
          ptx::st_v4(yr + v, normalize16<T>(xr[v], wsm[v], inv));
      }
    }
  }
  if (!load_ok) {
    // A copy never landed: record it, then wait (bounded) for the copies still in
    // flight so none lands in shared memory this CTA no longer owns.
    if (threadIdx.x == 0) {
      if (rp.state != nullptr) {
        if (atomicCAS(&rp.state->err_code, 0u, (unsigned)kStatusLoadTimeout) == 0u) {
          rp.state->err_call = call;
          if (rp.host_flag != nullptr) {
            *reinterpret_cast<volatile unsigned int*>(rp.host_flag) = (unsigned)kStatusLoadTimeout;
            __threadfence_system();
          }
        }
        atomicExch(&rp.state->abort, 1u);
      }
      for (int64_t kk = b; kk < issued; ++kk)
        mbar_wait_bounded(bar0 + 8u * (uint32_t)(kk % nslots), (uint32_t)((kk / nslots) & 1),
                          kLoadTimeoutNs);
    }
  }
  if (exchange) finish_launch(rp.state, call);
  flush_stats(a, ws, t_start);
}

// ---------------------------------------------------------------------------
// One-hop latency probe: a single thread bounces a counter between two GPUs.
// ---------------------------------------------------------------------------
__global__ void probe_roundtrip_kernel(unsigned long long* remote_slot,
                                       const unsigned long long* local_slot,
                                       unsigned long long seq, int iters, int initiator,
                                       unsigned long long timeout_ns, long long* out_ns,
                                       unsigned int* err_flag) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  const unsigned long long start = ptx::globaltimer();
  bool failed = false;
  for (int i = 1; i <= iters && !failed; ++i) {
    const unsigned long long v = (seq << 32) | (unsigned long long)i;
    if (initiator) ptx::st_relaxed_sys_u64(remote_slot, v);
    const unsigned long long t0 = ptx::globaltimer();
    while (ptx::ld_relaxed_sys_u64(local_slot) != v) {
      if (ptx::globaltimer() - t0 > timeout_ns) {
        failed = true;
        break;
      }
    }
    if (!initiator && !failed) ptx::st_relaxed_sys_u64(remote_slot, v);
  }
  const unsigned long long stop = ptx::globaltimer();
  if (failed) {
    if (err_flag) *err_flag = 1u;
    if (out_ns) *out_ns = -1;
  } else if (out_ns) {
    *out_ns = (long long)((stop - start) / (unsigned long long)(iters > 0 ? iters : 1));
  }
}

// ---------------------------------------------------------------------------
// Host side: variant table, plan, occupancy cache, launch.
// ---------------------------------------------------------------------------
namespace {

struct VariantShape {
  int vec, w, rows, block;
};
// Register kernels, selected by the number of 16-byte vectors per row, V: the
// first entry whose capacity 32 * w * vec >= V.
constexpr VariantShape kShapes[] = {
    {1, 1, 4, 256},   // V <= 32     (bf16 hl <= 256,   fp32 hl <= 128)
    {2, 1, 2, 256},   // V <= 64     (bf16 hl <= 512,   fp32 hl <= 256)
    {4, 1, 1, 256},   // V <= 128    (bf16 hl <= 1024,  fp32 hl <= 512)
    {4, 2, 1, 256},   // V <= 256    (bf16 hl <= 2048,  fp32 hl <= 1024)
    {4, 4, 1, 256},   // V <= 512    (bf16 hl <= 4096,  fp32 hl <= 2048)
    {4, 8, 1, 256},   // V <= 1024   (bf16 hl <= 8192,  fp32 hl <= 4096)
    {4, 16, 1, 512},  // V <= 2048   (bf16 hl <= 16384, fp32 hl <= 8192)
};
constexpr int kNumShapes = sizeof(kShapes) / sizeof(kShapes[0]);
constexpr int kGenericBlock = 256;

// Bulk kernels: (warps per CTA, stages per warp) x bound on rows per tile.
struct BulkShape {
  int warps, stages;
};
constexpr BulkShape kBulkShapes[] = {{4, 3}, {8, 3}, {16, 3}};
constexpr int kNumBulkShapes = sizeof(kBulkShapes) / sizeof(kBulkShapes[0]);
constexpr int kBulkRowBounds[] = {1, 2, 4, 8};
constexpr int kNumRowBounds = sizeof(kBulkRowBounds) / sizeof(kBulkRowBounds[0]);
constexpr int kNumBulk = kNumBulkShapes * kNumRowBounds;   // variant = base + shape * 4 + bound
constexpr uint32_t kBulkMaxRowBytes = 16384;          // one row must fit a stage
constexpr uint32_t kBulkSmemBudget = 216u * 1024u;    // dynamic smem of one CTA (1 CTA / SM)
constexpr uint64_t kBulkMinCallBytes = 48ull << 20;   // auto: bulk kernels from 48 MiB of x
// TP = 1 register kernels: tiles in flight per team. Measured on B200 (TP = 1,
// hidden 4096, 1..65536 rows): 3 is fastest for bf16 at every size and for fp32
// but at 4096 rows (4096 x 4096 bf16: 12.8 us at 3, 13.3 us at 4, 15.1 us at 6,
// which spills). With the fused residual add a buffer holds x and r: 2 tiles.
constexpr int kLocalDepths[] = {3, 4};
constexpr int kNumLocalDepths = sizeof(kLocalDepths) / sizeof(kLocalDepths[0]);
constexpr int kDefaultLocalDepth = 0;                 // index into kLocalDepths
// auto at TP = 1: bulk kernels from 256 MiB of x (the local kernel measured
// faster at 128 MiB, 45.3 vs 46.0 us; slower at 512 MiB, 169.6 vs 164.8 us)
constexpr uint64_t kBulkMinLocalCallBytes = 256ull << 20;
constexpr int kNumLocal = kNumShapes * kNumLocalDepths;
constexpr int kLocalResDepth = 2;
// fused residual add, bulk kernels: 4 warps x 3 stages, stage = x tile + residual tile
constexpr int kBulkResWarps = 4, kBulkResStages = 3;
constexpr uint32_t kBulkResMaxRowBytes = 8192;
// Batch kernels: 8 warps with 2 CTAs per SM (dynamic shared memory of a CTA at
// most kBatchSmem2), or 16 warps with 1 CTA per SM (at most kBatchSmem1).
constexpr int kBatchWarps[] = {8, 16};
constexpr int kNumBatch = sizeof(kBatchWarps) / sizeof(kBatchWarps[0]);
constexpr uint32_t kBatchSmem2 = 100u * 1024u;
constexpr uint32_t kBatchSmem1 = 200u * 1024u;
constexpr uint32_t kBatchMaxRowBytes = 16384;
constexpr uint32_t kBatchBytes = 16384;      // target bytes of x per batch
constexpr uint32_t kBatchMinBytes = 4096;    // smaller batches only to give every CTA work
constexpr int kBatchLag = 2;
// occupancy-cache slots: register, generic, bulk, local, then the residual
// kernels: local, bulk, generic; then the batch kernels
constexpr int kSlotLocalRes = kNumShapes + 1 + kNumBulk + kNumLocal;
constexpr int kSlotBulkRes = kSlotLocalRes + kNumShapes;
constexpr int kSlotGenericRes = kSlotBulkRes + kNumRowBounds;
constexpr int kSlotBatch = kSlotGenericRes + 1;
constexpr int kSlotResident = kSlotBatch + kNumBatch;
constexpr int kSlots = kSlotResident + kNumShapes;

using KernelFn = void (*)(const KArgs);

template <typename T>
struct KernelTable {
  static constexpr KernelFn vec[kNumShapes] = {
      tp_rmsnorm_vec_kernel<T, 1, 1, 4, 256, 2>, tp_rmsnorm_vec_kernel<T, 2, 1, 2, 256, 2>,
      tp_rmsnorm_vec_kernel<T, 4, 1, 1, 256, 2>, tp_rmsnorm_vec_kernel<T, 4, 2, 1, 256, 2>,
      tp_rmsnorm_vec_kernel<T, 4, 4, 1, 256, 2>, tp_rmsnorm_vec_kernel<T, 4, 8, 1, 256, 2>,
      tp_rmsnorm_vec_kernel<T, 4, 16, 1, 512, 1>,
  };
  static constexpr KernelFn bulk[kNumBulk] = {
      tp_rmsnorm_bulk_kernel<T, 4, 3, 1>,  tp_rmsnorm_bulk_kernel<T, 4, 3, 2>,
      tp_rmsnorm_bulk_kernel<T, 4, 3, 4>,  tp_rmsnorm_bulk_kernel<T, 4, 3, 8>,
      tp_rmsnorm_bulk_kernel<T, 8, 3, 1>,  tp_rmsnorm_bulk_kernel<T, 8, 3, 2>,
      tp_rmsnorm_bulk_kernel<T, 8, 3, 4>,  tp_rmsnorm_bulk_kernel<T, 8, 3, 8>,
      tp_rmsnorm_bulk_kernel<T, 16, 3, 1>, tp_rmsnorm_bulk_kernel<T, 16, 3, 2>,
      tp_rmsnorm_bulk_kernel<T, 16, 3, 4>, tp_rmsnorm_bulk_kernel<T, 16, 3, 8>,
  };
#define RTP_LOCAL(V, W, R, B, M) \
  rmsnorm_local_vec_kernel<T, V, W, R, B, M, 3>, rmsnorm_local_vec_kernel<T, V, W, R, B, M, 4>
  static constexpr KernelFn local[kNumLocal] = {
      RTP_LOCAL(1, 1, 4, 256, 2), RTP_LOCAL(2, 1, 2, 256, 2), RTP_LOCAL(4, 1, 1, 256, 2),
      RTP_LOCAL(4, 2, 1, 256, 2), RTP_LOCAL(4, 4, 1, 256, 2), RTP_LOCAL(4, 8, 1, 256, 2),
      RTP_LOCAL(4, 16, 1, 512, 1),
  };
#undef RTP_LOCAL
#define RTP_LOCAL_RES(V, W, R, B, M) rmsnorm_local_vec_kernel<T, V, W, R, B, M, kLocalResDepth, true>
  static constexpr KernelFn local_res[kNumShapes] = {
      RTP_LOCAL_RES(1, 1, 4, 256, 2), RTP_LOCAL_RES(2, 1, 2, 256, 2), RTP_LOCAL_RES(4, 1, 1, 256, 2),
      RTP_LOCAL_RES(4, 2, 1, 256, 2), RTP_LOCAL_RES(4, 4, 1, 256, 2), RTP_LOCAL_RES(4, 8, 1, 256, 2),
      RTP_LOCAL_RES(4, 16, 1, 512, 1),
  };
#undef RTP_LOCAL_RES
  static constexpr KernelFn bulk_res[kNumRowBounds] = {
      tp_rmsnorm_bulk_kernel<T, kBulkResWarps, kBulkResStages, 1, true>,
      tp_rmsnorm_bulk_kernel<T, kBulkResWarps, kBulkResStages, 2, true>,
      tp_rmsnorm_bulk_kernel<T, kBulkResWarps, kBulkResStages, 4, true>,
      tp_rmsnorm_bulk_kernel<T, kBulkResWarps, kBulkResStages, 8, true>,
  };
  static constexpr KernelFn generic = tp_rmsnorm_generic_kernel<T, kGenericBlock>;
  static constexpr KernelFn generic_res = tp_rmsnorm_generic_kernel<T, kGenericBlock, true>;
  static constexpr KernelFn batch[kNumBatch] = {tp_rmsnorm_batch_kernel<T, 8>,
                                                tp_rmsnorm_batch_kernel<T, 16>};
#define RTP_RESIDENT(V, W, R, B, M) tp_rmsnorm_vec_resident_kernel<T, V, W, R, B, M, kResidentDepth>
  static constexpr KernelFn resident[kNumShapes] = {
      RTP_RESIDENT(1, 1, 4, 256, 2), RTP_RESIDENT(2, 1, 2, 256, 2), RTP_RESIDENT(4, 1, 1, 256, 2),
      RTP_RESIDENT(4, 2, 1, 256, 2), RTP_RESIDENT(4, 4, 1, 256, 2), RTP_RESIDENT(4, 8, 1, 256, 2),
      RTP_RESIDENT(4, 16, 1, 512, 1),
  };
#undef RTP_RESIDENT
  static KernelFn get(int variant) {
    if (variant == kGenericRes) return generic_res;
    if (variant < 0) return generic;
    if (variant >= kResidentBase) return resident[variant - kResidentBase];
    if (variant >= kBatchBase) return batch[variant - kBatchBase];
    if (variant >= kBulkResBase) return bulk_res[variant - kBulkResBase];
    if (variant >= kLocalResBase) return local_res[variant - kLocalResBase];
    if (variant >= kLocalBase) return local[variant - kLocalBase];
    if (variant >= kBulkBase) return bulk[variant - kBulkBase];
    return vec[variant];
  }
};

KernelFn kernel_for(int dtype, int variant) {
  switch (dtype) {
    case kF32:
      return KernelTable<float>::get(variant);
    case kBF16:
      return KernelTable<__nv_bfloat16>::get(variant);
    default:
      return KernelTable<__half>::get(variant);
  }
}

int slot_of(int variant) {
  if (variant == kGenericRes) return kSlotGenericRes;
  if (variant >= kResidentBase) return kSlotResident + (variant - kResidentBase);
  if (variant >= kBatchBase) return kSlotBatch + (variant - kBatchBase);
  if (variant < 0) return kNumShapes;
  if (variant >= kBulkResBase) return kSlotBulkRes + (variant - kBulkResBase);
  if (variant >= kLocalResBase) return kSlotLocalRes + (variant - kLocalResBase);
  if (variant >= kLocalBase) return kNumShapes + 1 + kNumBulk + (variant - kLocalBase);
  if (variant >= kBulkBase) return kNumShapes + 1 + (variant - kBulkBase);
  return variant;
}

std::atomic<int> g_family{kFamilyAuto};
std::atomic<bool> g_dependent_launch{true};
std::atomic<int> g_push_mode{kPushPacked};

constexpr int kMaxDevices = 64;
// Per device/dtype/variant: (dynamic smem bytes << 32) | resident CTAs of the
// last occupancy query; 0 = none yet. Bulk kernels also get their max dynamic
// shared memory raised once (bit 31 of g_attr_set).
std::atomic<unsigned long long> g_resident[kMaxDevices][3][kSlots];
std::atomic<unsigned int> g_attr_set[kMaxDevices][3][kSlots];

std::atomic<int> g_sms[kMaxDevices];

int sm_count(int device, cudaError_t* err) {
  *err = cudaSuccess;
  const bool cacheable = device >= 0 && device < kMaxDevices;
  if (cacheable) {
    const int c = g_sms[device].load(std::memory_order_relaxed);
    if (c > 0) return c;
  }
  int sms = 0;
  *err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  if (*err != cudaSuccess) return 0;
  if (cacheable) g_sms[device].store(sms, std::memory_order_relaxed);
  return sms;
}

int resident_ctas(int device, int dtype, const VariantDesc& v, cudaError_t* err) {
  *err = cudaSuccess;
  const int slot = slot_of(v.id);
  const bool cacheable = device >= 0 && device < kMaxDevices;
  const void* fn = reinterpret_cast<const void*>(kernel_for(dtype, v.id));
  if (cacheable) {
    const unsigned long long c = g_resident[device][dtype][slot].load(std::memory_order_relaxed);
    if (c != 0ull && (unsigned)(c >> 32) == v.smem_bytes) return (int)(c & 0xFFFFFFFFull);
  }
  if (v.smem_bytes > 48u * 1024u && (!cacheable || g_attr_set[device][dtype][slot].load() == 0u)) {
    *err = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)kBulkSmemBudget);
    if (*err != cudaSuccess) return 0;
    // the whole unified L1/shared array as shared memory, so that the occupancy
    // the grid is sized by (one resident wave) is the occupancy the launch gets
    *err = cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout,
                                (int)cudaSharedmemCarveoutMaxShared);
    if (*err != cudaSuccess) return 0;
    if (cacheable) g_attr_set[device][dtype][slot].store(1u);
  }
  int per_sm = 0, sms = 0;
  *err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, v.block_threads,
                                                       (size_t)v.smem_bytes);
  if (*err != cudaSuccess) return 0;
  *err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  if (*err != cudaSuccess) return 0;
  const int total = per_sm * sms;
  if (cacheable && total > 0)
    g_resident[device][dtype][slot].store(((unsigned long long)v.smem_bytes << 32) | (unsigned)total,
                                          std::memory_order_relaxed);
  return total;
}

}  // namespace

void set_family(int family) { g_family.store(family); }
int get_family() { return g_family.load(); }
void set_dependent_launch(bool enable) { g_dependent_launch.store(enable); }
bool get_dependent_launch() { return g_dependent_launch.load(); }
void set_push_mode(int mode) { g_push_mode.store(mode); }
int get_push_mode() { return g_push_mode.load(); }

int elem_bytes(int dtype) { return dtype == kF32 ? 4 : 2; }

namespace {
// Tuning overrides from the environment, read once per process (-1 = unset):
// RMSNORM_TP_BULK_STAGE_BYTES (1024..16384), RMSNORM_TP_BULK_SCHEDULE (0..3),
// RMSNORM_TP_LOCAL_DEPTH (3 or 4).
struct Tuning {
  long stage_bytes = -1;
  int schedule = -1;
  int local_depth = -1;   // index into kLocalDepths
  // batch kernels: RMSNORM_TP_BATCH_BYTES (target bytes per batch, 1024..65536),
  // RMSNORM_TP_BATCH_MIN_BYTES (1024..65536), RMSNORM_TP_BATCH_LAG (1..6),
  // RMSNORM_TP_BATCH_CTAS (CTAs per SM: 1 or 2), RMSNORM_TP_BATCH_SLOTS (3..8)
  long batch_bytes = -1, batch_min_bytes = -1;
  int batch_lag = -1, batch_ctas = -1, batch_slots = -1;
  Tuning() {
    auto env_long = [](const char* name, long lo, long hi, long& out) {
      if (const char* env = std::getenv(name)) {
        const long v = std::atol(env);
        if (v >= lo && v <= hi) out = v;
      }
    };
    long v = -1;
    env_long("RMSNORM_TP_BATCH_BYTES", 1024, 65536, batch_bytes);
    env_long("RMSNORM_TP_BATCH_MIN_BYTES", 1024, 65536, batch_min_bytes);
    if (env_long("RMSNORM_TP_BATCH_LAG", 1, 6, v), v > 0) batch_lag = (int)v;
    v = -1;
    if (env_long("RMSNORM_TP_BATCH_CTAS", 1, 2, v), v > 0) batch_ctas = (int)v;
    v = -1;
    if (env_long("RMSNORM_TP_BATCH_SLOTS", 3, kBatchMaxSlots, v), v > 0) batch_slots = (int)v;
    if (const char* env = std::getenv("RMSNORM_TP_BULK_STAGE_BYTES")) {
      const long v = std::atol(env);
      if (v >= 1024 && v <= 16384) stage_bytes = v;
    }
    if (const char* env = std::getenv("RMSNORM_TP_BULK_SCHEDULE")) {
      const int v = std::atoi(env);
      if (v >= 0 && v <= 3) schedule = v;
    }
    if (const char* env = std::getenv("RMSNORM_TP_LOCAL_DEPTH")) {
      const int v = std::atoi(env);
      for (int d = 0; d < kNumLocalDepths; ++d)
        if (kLocalDepths[d] == v) local_depth = d;
    }
  }
};
const Tuning& tuning() {
  static const Tuning t;
  return t;
}
}  // namespace

namespace {
// Row-size dependent normalisation order of the bulk kernels (KArgs::schedule),
// as measured on B200 (TP = 1, 512 MiB of x): 8 KB rows one after another;
// 4 KB rows per-row reduction, interleaved normalisation; 2 KB rows one after
// another; <= 1 KB rows interleaved.
int bulk_schedule(uint32_t row_bytes) {
  if (row_bytes >= 8192u) return 3;
  if (row_bytes >= 4096u) return 1;
  if (row_bytes >= 2048u) return 3;
  return 0;
}

// Kernels of the fused residual add. TP = 1: the local register kernel (two
// tiles of x and r in flight per team) unless the call is large or the bulk
// family is forced. With an exchange: the bulk kernel (there is no register
// kernel with both an exchange and a residual), for rows of up to 8 KB, whose
// x + r stages fit shared memory; the generic kernel otherwise.
VariantDesc choose_residual_variant(int64_t hl, int dtype, bool vec_ok, int tp, int64_t rows,
                                    int family) {
  const int eb = elem_bytes(dtype);
  const uint32_t row_bytes = vec_ok ? (uint32_t)(hl * eb) : 0u;
  const uint64_t x_bytes = (uint64_t)rows * (uint64_t)hl * (uint64_t)eb;
  const bool bulk_fits = vec_ok && row_bytes <= kBulkResMaxRowBytes;
  const bool want_bulk =
      bulk_fits && (tp > 1 || family == kFamilyBulk ||
                    (family == kFamilyAuto && x_bytes >= kBulkMinLocalCallBytes));
  if (want_bulk) {
    const uint32_t w_bytes = (row_bytes + 127u) & ~127u;
    int max_rows = tp > 1 ? 32 / tp : 32;
    if (max_rows > kBulkRowBounds[kNumRowBounds - 1]) max_rows = kBulkRowBounds[kNumRowBounds - 1];
    int tile_rows = (int)(8192u / row_bytes);   // 8 KB of x (and 8 KB of r) per stage
    if (tile_rows > max_rows) tile_rows = max_rows;
    if (tile_rows < 1) tile_rows = 1;
    int bound = 0;
    while (kBulkRowBounds[bound] < tile_rows) ++bound;
    const uint32_t stage = 2u * (((uint32_t)tile_rows * row_bytes + 127u) & ~127u);
    const uint32_t smem = w_bytes + (uint32_t)(kBulkResWarps * kBulkResStages) * stage;  // <= 200 KB
    return VariantDesc{kBulkResBase + bound, kBulkResStages, 1, tile_rows, kBulkResWarps * 32,
                       stage, smem, 1, bulk_schedule(row_bytes), kBulkResStages};
  }
  if (vec_ok && tp == 1) {
    const int64_t V = hl * eb / 16;
    for (int i = 0; i < kNumShapes; ++i)
      if (V <= 32ll * kShapes[i].w * kShapes[i].vec)
        return VariantDesc{kLocalResBase + i, kShapes[i].vec, kShapes[i].w, kShapes[i].rows,
                           kShapes[i].block, 0u, 0u, 0, 0, kLocalResDepth};
  }
  return VariantDesc{kGenericRes, 0, kGenericBlock / 32, 1, kGenericBlock, 0u, 0u, 0, 0, 1};
}
}  // namespace

namespace {
// Batch kernel shape for rows of row_bytes (<= kBatchMaxRowBytes): rows per
// batch, ring slots, lag. Batches of ~kBatchBytes of x, made smaller (down to
// kBatchMinBytes) while the call has fewer than two batches per CTA, so that
// small calls still spread over the chip and pipeline within a CTA.
VariantDesc batch_variant(uint32_t row_bytes, int64_t rows, int sms) {
  const Tuning& t = tuning();
  const int ctas_per_sm = t.batch_ctas > 0 ? t.batch_ctas : 2;
  const int idx = ctas_per_sm == 2 ? 0 : 1;
  const uint32_t budget = ctas_per_sm == 2 ? kBatchSmem2 : kBatchSmem1;
  const uint32_t w_bytes = (row_bytes + 127u) & ~127u;
  const uint32_t target = t.batch_bytes > 0 ? (uint32_t)t.batch_bytes : kBatchBytes;
  const uint32_t min_bytes = t.batch_min_bytes > 0 ? (uint32_t)t.batch_min_bytes : kBatchMinBytes;
  int bR = (int)(target / row_bytes);
  if (bR > kBatchMaxRows) bR = kBatchMaxRows;
  if (bR < 1) bR = 1;
  const int64_t ctas = (int64_t)sms * ctas_per_sm;
  while (bR > 1 && (rows + bR - 1) / bR < 2 * ctas && (uint32_t)bR * row_bytes > min_bytes) bR /= 2;
  // at least 3 slots: a refill is then issued before the batch it fetches is awaited
  while (bR > 1 && (budget - w_bytes) / (((uint32_t)bR * row_bytes + 127u) & ~127u) < 3u) bR /= 2;
  const uint32_t slot = ((uint32_t)bR * row_bytes + 127u) & ~127u;
  int nslots = (int)((budget - w_bytes) / slot);
  if (nslots > kBatchMaxSlots) nslots = kBatchMaxSlots;
  if (t.batch_slots > 0 && t.batch_slots < nslots) nslots = t.batch_slots;
  const int lag = t.batch_lag > 0 ? t.batch_lag : kBatchLag;
  return VariantDesc{kBatchBase + idx, nslots, kBatchWarps[idx], bR, kBatchWarps[idx] * 32, slot,
                     w_bytes + (uint32_t)nslots * slot, lag, 0, nslots};
}
}  // namespace

VariantDesc choose_variant(int64_t hl, int dtype, bool aligned, int tp, int64_t rows, int family,
                           bool residual, int sms) {
  const int eb = elem_bytes(dtype);
  const bool vec_ok = aligned && hl > 0 && ((hl * eb) % 16 == 0);
  if (family == kFamilyAuto) family = get_family();
  if (residual) {
    if (family == kFamilyBatch) family = kFamilyAuto;   // no batch kernel with a residual
    return choose_residual_variant(hl, dtype, vec_ok, tp, rows, family);
  }
  // batch kernels: when the family is forced (aligned rows that fit a slot)
  if (vec_ok && (uint64_t)hl * eb <= kBatchMaxRowBytes && family == kFamilyBatch) {
    const VariantDesc v = batch_variant((uint32_t)(hl * eb), rows, sms);
    if (v.depth >= 3) return v;
  }
  // bulk kernels for large calls (>= kBulkMinCallBytes of x per rank with an
  // exchange, >= kBulkMinLocalCallBytes at TP = 1), register kernels below
  // that, where their lower fixed cost wins (measured on B200: with an
  // exchange, register faster at 32 MiB, bulk faster from 64 MiB). Rows of 16 KB
  // at TP = 1 (one-row tiles, 4 warps per SM) stay on the register kernel, which
  // measured faster there at every size; with an exchange the bulk kernel wins.
  const uint64_t x_bytes = (uint64_t)rows * (uint64_t)hl * (uint64_t)eb;
  const bool large = tp > 1 ? x_bytes >= kBulkMinCallBytes
                            : x_bytes >= kBulkMinLocalCallBytes && (uint64_t)hl * eb < kBulkMaxRowBytes;
  const bool want_bulk = family == kFamilyBulk || (family == kFamilyAuto && large);
  if (vec_ok && want_bulk && (uint64_t)hl * eb <= kBulkMaxRowBytes) {
    const uint32_t row_bytes = (uint32_t)(hl * eb);
    const uint32_t w_bytes = (row_bytes + 127u) & ~127u;
    // one lane per (row, rank) in the exchange; at most 8 rows per tile
    int max_rows = tp > 1 ? 32 / tp : 32;
    if (max_rows > kBulkRowBounds[kNumRowBounds - 1]) max_rows = kBulkRowBounds[kNumRowBounds - 1];
    // tiles of 8 KB of x; 16 KB for 8 KB rows at TP = 1 (measured on B200 at
    // 512 MiB of x: 99% of the copy peak vs 85% with one-row tiles)
    uint32_t target = 8192u;
    int schedule = bulk_schedule(row_bytes);
    // 2-row 16 KB tiles for 8 KB rows win at TP = 1 only; with an exchange,
    // one-row 8 KB tiles measured faster (TP 2, 65536 rows: 98% vs 83% of the copy peak)
    if (row_bytes >= 8192u && tp == 1) target = 16384u;
    if (tuning().stage_bytes > 0) target = (uint32_t)tuning().stage_bytes;
    if (tuning().schedule >= 0) schedule = tuning().schedule;
    if (target < row_bytes) target = row_bytes;
    int tile_rows = (int)(target / row_bytes);
    if (tile_rows > max_rows) tile_rows = max_rows;
    if (tile_rows < 1) tile_rows = 1;
    int bound = 0;
    while (kBulkRowBounds[bound] < tile_rows) ++bound;
    const uint32_t stage = ((uint32_t)tile_rows * row_bytes + 127u) & ~127u;
    for (int i = kNumBulkShapes - 1; i >= 0; --i) {
      const uint32_t smem = w_bytes + (uint32_t)kBulkShapes[i].warps * kBulkShapes[i].stages * stage;
      if (smem <= kBulkSmemBudget)
        return VariantDesc{kBulkBase + i * kNumRowBounds + bound, kBulkShapes[i].stages, 1,
                           tile_rows, kBulkShapes[i].warps * 32, stage, smem, 1, schedule,
                           kBulkShapes[i].stages};
    }
  }
  if (vec_ok) {
    const int64_t V = hl * eb / 16;
    for (int i = 0; i < kNumShapes; ++i) {
      const int64_t cap = 32ll * kShapes[i].w * kShapes[i].vec;
      if (V > cap) continue;
      // without an exchange (TP = 1): the local kernel, all buffers loading
      int id = i, in_flight = 3;
      if (tp == 1) {
        const int depth = tuning().local_depth >= 0 ? tuning().local_depth : kDefaultLocalDepth;
        id = kLocalBase + i * kNumLocalDepths + depth;
        in_flight = kLocalDepths[depth];
      }
      return VariantDesc{id, kShapes[i].vec, kShapes[i].w, kShapes[i].rows, kShapes[i].block, 0u, 0u,
                         0, 0, in_flight};
    }
  }
  return VariantDesc{-1, 0, kGenericBlock / 32, 1, kGenericBlock, 0u, 0u, 0, 0, 1};
}

VariantDesc finalize_variant(const VariantDesc& v, int tp, int64_t rows, int resident_ctas) {
  if (tp < 2 || v.id < 0 || v.id >= kNumShapes || get_family() == kFamilyRegister) return v;
  // decode-sized calls only: for the 4096-row benchmark call the rotating kernel
  // measured faster on B200 at every group size (TP 2 / 4 / 8: 11.5 / 10.0 / 9.4
  // us against 12.0 / 10.6 / 9.8 us per call)
  if (rows > kResidentMaxRows) return v;
  const int64_t teams = (int64_t)resident_ctas * (v.block_threads / 32 / v.team_warps);
  const int64_t tiles = (rows + v.rows_per_tile - 1) / v.rows_per_tile;
  if (tiles > teams * kResidentDepth) return v;
  VariantDesc r = v;
  r.id = kResidentBase + v.id;
  r.depth = (int)((tiles + teams - 1) / (teams > 0 ? teams : 1));
  if (r.depth < 1) r.depth = 1;
  return r;
}

Plan plan_for(const VariantDesc& v, int64_t rows, int resident_ctas) {
  Plan p{};
  p.variant = v.id;
  p.vec_per_lane = v.vec_per_lane;
  p.team_warps = v.team_warps;
  p.rows_per_tile = v.rows_per_tile;
  p.block_threads = v.block_threads;
  p.depth = v.depth;
  p.teams_per_cta = v.block_threads / 32 / v.team_warps;
  p.tiles = rows > 0 ? (rows + v.rows_per_tile - 1) / v.rows_per_tile : 0;
  const int64_t need = (p.tiles + p.teams_per_cta - 1) / p.teams_per_cta;
  int64_t grid = need < (int64_t)resident_ctas ? need : (int64_t)resident_ctas;
  if (grid < 1) grid = 1;
  p.grid = (int)grid;
  return p;
}

cudaError_t launch_forward(const KArgs& a_in, int dtype, int device, int grid_y,
                           cudaStream_t stream, Plan* plan_out) {
  const int nranks = a_in.emulated ? grid_y : 1;
  const bool residual = a_in.rp[0].res != nullptr;
  bool aligned = true;
  for (int r = 0; r < nranks; ++r) {
    const uintptr_t bits = reinterpret_cast<uintptr_t>(a_in.rp[r].x) |
                           reinterpret_cast<uintptr_t>(a_in.rp[r].out) |
                           reinterpret_cast<uintptr_t>(a_in.rp[r].w) |
                           reinterpret_cast<uintptr_t>(a_in.rp[r].res);
    if (bits & 15u) aligned = false;
  }
  cudaError_t err = cudaSuccess;
  const int sms = sm_count(device, &err);
  if (err != cudaSuccess) return err;
  const VariantDesc v =
      choose_variant(a_in.hl, dtype, aligned, a_in.tp, a_in.rows, kFamilyAuto, residual, sms);
  int resident = resident_ctas(device, dtype, v, &err);
  if (err != cudaSuccess) return err;
  if (grid_y > 1) resident /= grid_y;
  if (resident < 1) return cudaErrorCooperativeLaunchTooLarge;
  VariantDesc v2 = finalize_variant(v, a_in.tp, a_in.rows, resident);
  if (v2.id != v.id) {   // the resident kernel's own occupancy sizes its grid
    int r2 = resident_ctas(device, dtype, v2, &err);
    if (err != cudaSuccess) return err;
    if (grid_y > 1) r2 /= grid_y;
    if (r2 < resident) v2 = v;   // fewer resident CTAs: keep the rotating kernel
  }
  const Plan p = plan_for(v2, a_in.rows, resident);
  if (plan_out) *plan_out = p;
  KArgs a = a_in;
  a.tile_rows = v.rows_per_tile;
  a.stage_bytes = v.stage_bytes;
  a.lag = v.lag;
  a.schedule = v.schedule;
  a.depth = v.depth;
  a.push_mode = get_push_mode();
  const void* fn = reinterpret_cast<const void*>(kernel_for(dtype, v2.id));
  void* args[] = {&a};
  const dim3 grid((unsigned)p.grid, (unsigned)grid_y);
  const dim3 block((unsigned)p.block_threads);
  if (grid_y > 1) return cudaLaunchCooperativeKernel(fn, grid, block, args, v.smem_bytes, stream);
  if (!get_dependent_launch()) return cudaLaunchKernel(fn, grid, block, args, v.smem_bytes, stream);
  // Programmatic dependent launch: the kernel may be scheduled while the
  // stream's previous kernel finishes; its first instruction (griddepcontrol.wait)
  // holds it until that kernel has completed and its writes are visible.
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = v.smem_bytes;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelExC(&cfg, fn, args);
}

cudaError_t launch_probe(unsigned long long* remote_slot, unsigned long long* local_slot,
                         unsigned long long seq, int iters, int initiator,
                         unsigned long long timeout_ns, long long* out_ns,
                         unsigned int* err_flag, cudaStream_t stream) {
  probe_roundtrip_kernel<<<1, 32, 0, stream>>>(remote_slot, local_slot, seq, iters, initiator,
                                               timeout_ns, out_ns, err_flag);
  return cudaPeekAtLastError();
}

}  // namespace rtp
