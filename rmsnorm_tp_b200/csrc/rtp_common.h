// Shared host/device definitions of the fused tensor-parallel RMSNorm.
//
// Everything here is plain arithmetic that both the CUDA kernels and the host
// C-ABI use, so the host unit tests exercise exactly the code the device runs:
//   * the per-rank device state (generation counter, completion counter, error
//     record),
//   * the generation -> (mailbox buffer, tag) mapping that replaces the
//     reference's `int generation` kernel argument and `>=` poll
//     (reference csrc/rmsnorm_tp.cu:61, :114, :128),
//   * the packed 64-bit mailbox word {partial sum, tag},
//   * the mailbox slot layout (reference csrc/bindings.cpp:26-33 keeps
//     float sums[tp][rows] + int gen[tp][rows]; here one u64 per slot, two
//     generation buffers, rows strided by num_max_rows),
//   * the row -> team mapping of the launch plan.
#pragma once

#include <stdint.h>
#include <string.h>

#if defined(__CUDACC__)
#define RTP_HD __host__ __device__ __forceinline__
#else
#define RTP_HD static inline
#endif

namespace rtp {

constexpr int kMaxTP = 8;              // reference common.hpp:9 (MAX_TP_SIZE)
constexpr int kHandleBytes = 128;      // reference common.hpp:10 (HANDLE_SIZE)
constexpr uint32_t kHandleMagic = 0x42505452u;  // "RTPB"
constexpr uint32_t kHandleVersion = 1u;

// Device-side failure codes recorded in DeviceState::err_code and mirrored
// into the host-mapped flag word.
enum DeviceStatus : uint32_t {
  kStatusOk = 0,
  kStatusTimeout = 1,   // a peer's partial sum did not arrive within the limit
  kStatusAborted = 2,   // gave up because another CTA on this GPU timed out
  kStatusLoadTimeout = 3,  // a bulk copy into shared memory did not complete in time
};

// Per-rank state in local device memory (never mapped to peers).
// `call` holds kGenUnit x (the generation of the next launch), plus, while a
// one-generation launch (forward, linear) runs, the shares its CTAs have added
// so far: at its end CTA 0 adds kGenUnit - (grid - 1) and every other CTA adds
// 1 (fire-and-forget, no returning atomic), so a finished launch of any grid
// size advances `call` by exactly kGenUnit. A CTA reads `call` before it adds
// its own share, so the shares it can see leave out its own: with CTA 0's they
// sum to at most kGenUnit - 1, without it to at most grid - 1 (grids stay far
// below kGenUnit CTAs), and call >> kGenShift is the launch's generation. A
// two-generation launch (backward) cannot split its advance that way (one share
// alone would reach a unit), so its last CTA -- found by a returning atomic on
// `done` -- stores the advanced value. The next launch reads `call` only after
// this grid has completed.
constexpr int kGenShift = 20;
constexpr unsigned long long kGenUnit = 1ull << kGenShift;
constexpr unsigned long long kGenMax = (1ull << (64 - kGenShift)) - 1ull;   // largest generation

struct alignas(64) DeviceState {
  unsigned long long call;      // kGenUnit x generation of the next launch (+ running shares)
  unsigned int done;            // CTAs of a running two-generation launch that have finished
  unsigned int abort;           // set once any CTA gave up; the rest give up fast
  unsigned int err_code;        // first failure (DeviceStatus), set with atomicCAS
  unsigned int err_src;         // source rank whose partial never arrived
  long long err_row;            // row that timed out
  unsigned int err_expected;    // tag that was awaited
  unsigned int err_seen;        // tag found in the slot when the wait ended
  unsigned long long err_call;  // generation of the failing launch
  unsigned long long reserved[3];
};

// ---------------------------------------------------------------------------
// Generation arithmetic.
//
// Call number `g` (a 64-bit count of launches, identical on every rank because
// every rank launches the same sequence) selects
//   buffer(g) = g & 1                 -- double buffer: a rank that has finished
//                                        call g may already push call g+1 while a
//                                        slow peer still reads call g's slots;
//                                        it cannot reach call g+2 before that
//                                        peer has pushed g+1, i.e. finished g.
//   tag(g)    = 1 + g mod (2^32 - 1)  -- never 0 (a zeroed mailbox never matches)
//                                        and tag(g) != tag(g+2) at every g, across
//                                        the 32-bit wrap included.
// The poll tests the tag for EQUALITY, so a stale slot from call g-2 (same
// buffer) is never taken for call g, unlike the reference's `< generation`
// test (rmsnorm_tp.cu:128), which also accepts newer generations.
// ---------------------------------------------------------------------------
// The device counter's share of CTA `cta` of a one-generation launch of `grid`
// CTAs, and the generation a counter value holds (see DeviceState).
RTP_HD uint64_t gen_share(uint32_t cta, uint32_t grid) {
  return cta == 0u ? kGenUnit - (uint64_t)(grid - 1u) : 1ull;
}
RTP_HD uint64_t gen_of(uint64_t counter) { return counter >> kGenShift; }

RTP_HD uint32_t tag_of(uint64_t g) { return (uint32_t)(g % 0xFFFFFFFFull) + 1u; }
RTP_HD uint32_t buffer_of(uint64_t g) { return (uint32_t)(g & 1ull); }

RTP_HD uint32_t f32_bits(float v) {
#if defined(__CUDA_ARCH__)
  return __float_as_uint(v);
#else
  uint32_t u;
  memcpy(&u, &v, 4);
  return u;
#endif
}
RTP_HD float bits_f32(uint32_t u) {
#if defined(__CUDA_ARCH__)
  return __uint_as_float(u);
#else
  float v;
  memcpy(&v, &u, 4);
  return v;
#endif
}

// One mailbox word: high 32 bits = tag, low 32 bits = fp32 partial sum of squares.
// A naturally aligned 64-bit store is single-copy atomic, so a reader that sees
// the tag also sees the value: no separate flag and no release/acquire pair.
RTP_HD uint64_t pack_slot(float partial, uint32_t tag) {
  return ((uint64_t)tag << 32) | (uint64_t)f32_bits(partial);
}
RTP_HD uint32_t slot_tag(uint64_t w) { return (uint32_t)(w >> 32); }
RTP_HD float slot_value(uint64_t w) { return bits_f32((uint32_t)(w & 0xFFFFFFFFull)); }

// Mailbox of one rank: u64 slot[2 buffers][tp source ranks][num_max_rows].
RTP_HD uint64_t slot_index(uint32_t buf, int src, int tp, int64_t nmax, int64_t row) {
  return ((uint64_t)buf * (uint64_t)tp + (uint64_t)src) * (uint64_t)nmax + (uint64_t)row;
}
RTP_HD uint64_t mailbox_slots(int tp, int64_t nmax) { return 2ull * (uint64_t)tp * (uint64_t)nmax; }

// ---------------------------------------------------------------------------
// Launch plan: which kernel variant handles a (rows, local_hidden, dtype) call
// and how rows map to "teams" (a team = team_warps warps sharing one row).
// Teams walk row tiles of rows_per_tile rows in a grid-stride loop; the grid is
// never larger than one resident wave, so every CTA of every rank is resident
// at once and the cross-GPU waits always make progress.
// ---------------------------------------------------------------------------
struct Plan {
  int variant;          // index in the variant table, -1 = generic (any alignment / width)
  int vec_per_lane;     // 16-byte vectors of one row held per lane
  int team_warps;       // warps that share one row
  int rows_per_tile;    // rows a team handles per step
  int block_threads;
  int teams_per_cta;
  int64_t tiles;        // ceil(rows / rows_per_tile)
  int grid;             // CTAs (x); <= resident capacity
  int depth;            // tiles in flight per team (bulk: stages per warp; generic: 1)
};

// First row of the tile a team handles at step `it`; rows [first, first + rows_per_tile)
RTP_HD int64_t tile_of(int64_t team_global, int64_t it, int64_t teams_total) {
  return team_global + it * teams_total;
}

// Output tile t of the fused row-parallel linear -> (m block, n block), for mt x nt
// tiles, tp owners of nbl column tiles each. Tiles go in groups of up to 16 m
// blocks: within a group the m block varies fastest, so the CTAs running at the
// same time share a few column slices of the weight (read once from HBM, then
// from L2) instead of streaming all of it per m block; the group's column index
// j is dealt over the owners (owner j % tp), so that consecutive tiles go to
// different ranks' receive buffers.
constexpr int64_t kLinGroupM = 16;
RTP_HD void linear_tile(int64_t t, int64_t mt, int64_t nt, int tp, int64_t nbl, int64_t* mb,
                        int64_t* nb) {
  const int64_t per_group = kLinGroupM * nt;
  const int64_t g = t / per_group;
  const int64_t left = mt - g * kLinGroupM;
  const int64_t gm = left < kLinGroupM ? left : kLinGroupM;
  const int64_t r = t - g * per_group;
  *mb = g * kLinGroupM + r % gm;
  const int64_t j = r / gm;
  *nb = (j % tp) * nbl + j / tp;
}

}  // namespace rtp
