// Host test of the mailbox protocol, built from the same header the CUDA
// kernels use (rmsnorm_tp_b200/csrc/rtp_common.h).
//
// 1. Generation arithmetic: tags are never 0, and a slot of the same buffer
//    left from any of the previous 10^6 same-buffer calls never carries the
//    current tag -- checked around 0, the 32-bit wrap and the tag period.
// 2. Slot packing and layout.
// 3. Simulation: tp threads play the ranks. Each call pushes {partial, tag}
//    into every peer's slot [buf][rank][row] and polls its own slots with the
//    equality test, exactly as the kernel's exchange does (relaxed atomics
//    stand in for relaxed system-scope accesses). Row counts vary from call to
//    call (stale slots), ranks run with random skew, the generation starts
//    just below the tag wrap. Every rank must read every peer's partial of the
//    current call and compute the same sum in rank order.
// 4. A rank that skips a call makes the others' waits run out (bounded), not
//    hang, and no rank ever sums a wrong partial.
// 5. Forward and backward calls mixed: a backward call takes two generations
//    (sum(x^2) in generation g, buffer g & 1, then sum(dy * w * x) in g + 1, the
//    other buffer) and pushes a row's second partial only after it has received
//    every peer's first partial of that row, as the backward kernel does. With
//    random skew, stale slots and the tag wrap, every partial read must be the
//    current call's. Built with -DRTP_PLANT_EARLY_SECOND_PUSH, the second
//    partial is pushed with the first (a planted protocol mistake): the program
//    must then report failures (the negative control of this check).
#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <random>
#include <thread>
#include <vector>

#include "rtp_common.h"

using namespace rtp;

static int g_failures = 0;
#define CHECK(cond, ...)                                 \
  do {                                                   \
    if (!(cond)) {                                       \
      std::printf("FAIL %s:%d: ", __FILE__, __LINE__);   \
      std::printf(__VA_ARGS__);                          \
      std::printf("\n");                                 \
      ++g_failures;                                      \
      return;                                            \
    }                                                    \
  } while (0)

static void test_generation() {
  const uint64_t P = 0xFFFFFFFFull;  // tag period
  const uint64_t starts[] = {0ull, (1ull << 32) - 3000000ull, P - 2000000ull, 2 * P - 1000000ull,
                             (1ull << 33) - 1000000ull, 0xFFFFFFFFFFull};
  for (uint64_t s : starts) {
    for (uint64_t g = s; g < s + 4000000ull; ++g) {
      const uint32_t t = tag_of(g);
      CHECK(t != 0u, "tag_of(%llu) == 0", (unsigned long long)g);
      CHECK(buffer_of(g) == (uint32_t)(g & 1ull), "buffer_of(%llu)", (unsigned long long)g);
      if (g >= s + 2) CHECK(tag_of(g - 2) != t, "tag_of(%llu) repeats after 2 calls", (unsigned long long)g);
    }
    // a stale slot of the same buffer from 2j calls back never aliases (j <= 10^6)
    const uint64_t g = s + 3000000ull;
    for (uint64_t j = 1; j <= 1000000ull; ++j)
      CHECK(tag_of(g - 2 * j) != tag_of(g), "alias at distance %llu", (unsigned long long)(2 * j));
  }
  CHECK(tag_of(P - 1) == 0xFFFFFFFFu && tag_of(P) == 1u, "tag wrap point");
  std::printf("PASS generation\n");
}

static void test_packing() {
  std::mt19937 rng(1);
  std::uniform_real_distribution<float> d(-1e30f, 1e30f);
  for (int i = 0; i < 100000; ++i) {
    const float v = (i % 7 == 0) ? 0.0f : d(rng);
    const uint32_t tag = (uint32_t)rng() | 1u;
    const uint64_t w = pack_slot(v, tag);
    CHECK(slot_tag(w) == tag, "tag round trip");
    CHECK(f32_bits(slot_value(w)) == f32_bits(v), "value round trip");
  }
  CHECK(slot_tag(pack_slot(-0.0f, 5u)) == 5u && f32_bits(slot_value(pack_slot(-0.0f, 5u))) == 0x80000000u,
        "negative zero");
  // layout: every (buf, src, row) maps to a distinct slot inside the mailbox
  for (int tp = 1; tp <= kMaxTP; ++tp) {
    const int64_t nmax = 37;
    std::vector<int> seen(mailbox_slots(tp, nmax), 0);
    for (uint32_t b = 0; b < 2; ++b)
      for (int s = 0; s < tp; ++s)
        for (int64_t r = 0; r < nmax; ++r) {
          const uint64_t i = slot_index(b, s, tp, nmax, r);
          CHECK(i < seen.size(), "slot out of range");
          seen[i] += 1;
        }
    for (int c : seen) CHECK(c == 1, "slot layout not a bijection at tp %d", tp);
  }
  std::printf("PASS packing\n");
}

struct Sim {
  int tp;
  int64_t nmax;
  std::vector<std::vector<std::atomic<uint64_t>>> mbox;  // [rank][slot]
  std::vector<int64_t> rows_of_call;
  uint64_t g0;
  std::atomic<int> errors{0};
  std::atomic<int> timeouts{0};
  std::atomic<long long> first_timeout_call{-1};

  Sim(int tp_, int64_t nmax_, int calls, uint64_t g0_, unsigned seed) : tp(tp_), nmax(nmax_), mbox(tp_), g0(g0_) {
    for (auto& m : mbox) {
      std::vector<std::atomic<uint64_t>> v(mailbox_slots(tp, nmax));
      for (auto& a : v) a.store(0, std::memory_order_relaxed);
      m.swap(v);
    }
    std::mt19937 rng(seed);
    for (int c = 0; c < calls; ++c) rows_of_call.push_back(1 + (int64_t)(rng() % (uint64_t)nmax));
  }

  static float partial(int rank, int call, int64_t row) {
    return (float)((rank + 1) * 1000 + (call % 997)) + 0.25f * (float)row;
  }

  // One rank's sequence of calls; skip_call >= 0 makes this rank skip that call.
  void run_rank(int rank, unsigned seed, int skip_call, double timeout_s) {
    std::mt19937 rng(seed);
    std::vector<int64_t> order;
    for (int c = 0; c < (int)rows_of_call.size(); ++c) {
      if (c == skip_call) continue;
      const uint64_t g = g0 + (uint64_t)c;
      const uint32_t buf = buffer_of(g), tag = tag_of(g);
      const int64_t R = rows_of_call[c];
      order.resize(R);
      for (int64_t r = 0; r < R; ++r) order[r] = r;
      std::shuffle(order.begin(), order.end(), rng);
      if (rng() % 8 == 0) std::this_thread::sleep_for(std::chrono::microseconds(rng() % 50));
      for (int64_t r : order)  // push phase
        for (int q = 0; q < tp; ++q)
          if (q != rank)
            mbox[q][slot_index(buf, rank, tp, nmax, r)].store(pack_slot(partial(rank, c, r), tag),
                                                             std::memory_order_relaxed);
      std::shuffle(order.begin(), order.end(), rng);
      for (int64_t r : order) {  // poll phase
        float S = 0.f, want = 0.f;
        for (int q = 0; q < tp; ++q) {
          want += partial(q, c, r);
          if (q == rank) {
            S += partial(rank, c, r);
            continue;
          }
          const auto t0 = std::chrono::steady_clock::now();
          uint64_t w;
          for (;;) {
            w = mbox[rank][slot_index(buf, q, tp, nmax, r)].load(std::memory_order_relaxed);
            if (slot_tag(w) == tag) break;
            if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > timeout_s) {
              timeouts.fetch_add(1);
              long long expected = -1;
              first_timeout_call.compare_exchange_strong(expected, c);
              return;  // this rank gives up, like the kernel's bounded wait
            }
            std::this_thread::yield();
          }
          S += slot_value(w);
        }
        if (f32_bits(S) != f32_bits(want)) errors.fetch_add(1);
      }
    }
  }
};

// Forward (one exchange) and backward (two exchanges) calls mixed.
struct MixedSim {
  int tp;
  int64_t nmax;
  std::vector<std::vector<std::atomic<uint64_t>>> mbox;  // [rank][slot]
  std::vector<int64_t> rows_of_call;
  std::vector<int> backward;                             // 1: the call is a backward
  std::vector<uint64_t> gen_of_call;                     // first generation of the call
  std::atomic<int> errors{0};
  std::atomic<int> timeouts{0};

  MixedSim(int tp_, int64_t nmax_, int calls, uint64_t g0, unsigned seed)
      : tp(tp_), nmax(nmax_), mbox(tp_) {
    for (auto& m : mbox) {
      std::vector<std::atomic<uint64_t>> v(mailbox_slots(tp, nmax));
      for (auto& a : v) a.store(0, std::memory_order_relaxed);
      m.swap(v);
    }
    std::mt19937 rng(seed);
    uint64_t g = g0;
    for (int c = 0; c < calls; ++c) {
      rows_of_call.push_back(1 + (int64_t)(rng() % (uint64_t)nmax));
      backward.push_back(rng() % 3 == 0 ? 1 : 0);
      gen_of_call.push_back(g);
      g += backward.back() ? 2u : 1u;
    }
  }

  static float partial(int rank, int call, int64_t row, int which) {
    return (float)((rank + 1) * 1000 + (call % 997)) + 0.25f * (float)row + 0.125f * (float)which;
  }

  void push(int rank, uint64_t g, int c, int64_t r, int which) {
    for (int q = 0; q < tp; ++q)
      if (q != rank)
        mbox[q][slot_index(buffer_of(g), rank, tp, nmax, r)].store(
            pack_slot(partial(rank, c, r, which), tag_of(g)), std::memory_order_relaxed);
  }

  // Sum of every rank's partial of row r in rank order; false on a timeout.
  bool poll(int rank, uint64_t g, int c, int64_t r, int which, double timeout_s) {
    float S = 0.f, want = 0.f;
    for (int q = 0; q < tp; ++q) {
      want += partial(q, c, r, which);
      if (q == rank) {
        S += partial(rank, c, r, which);
        continue;
      }
      const auto t0 = std::chrono::steady_clock::now();
      uint64_t w;
      for (;;) {
        w = mbox[rank][slot_index(buffer_of(g), q, tp, nmax, r)].load(std::memory_order_relaxed);
        if (slot_tag(w) == tag_of(g)) break;
        if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > timeout_s) {
          timeouts.fetch_add(1);
          return false;
        }
        std::this_thread::yield();
      }
      S += slot_value(w);
    }
    if (f32_bits(S) != f32_bits(want)) errors.fetch_add(1);
    return true;
  }

  void run_rank(int rank, unsigned seed, double timeout_s) {
    std::mt19937 rng(seed);
    std::vector<int64_t> order;
    for (int c = 0; c < (int)rows_of_call.size(); ++c) {
      const uint64_t g = gen_of_call[c];
      const int64_t R = rows_of_call[c];
      order.resize(R);
      for (int64_t r = 0; r < R; ++r) order[r] = r;
      if (rng() % 8 == 0) std::this_thread::sleep_for(std::chrono::microseconds(rng() % 50));
      std::shuffle(order.begin(), order.end(), rng);
      for (int64_t r : order) {
        push(rank, g, c, r, 0);
#ifdef RTP_PLANT_EARLY_SECOND_PUSH
        if (backward[c]) push(rank, g + 1, c, r, 1);   // planted: before the first exchange
#endif
      }
      std::shuffle(order.begin(), order.end(), rng);
      for (int64_t r : order) {
        if (!poll(rank, g, c, r, 0, timeout_s)) return;
#ifndef RTP_PLANT_EARLY_SECOND_PUSH
        if (backward[c]) push(rank, g + 1, c, r, 1);   // only after row r's first exchange
#endif
      }
      if (backward[c]) {
        std::shuffle(order.begin(), order.end(), rng);
        for (int64_t r : order)
          if (!poll(rank, g + 1, c, r, 1, timeout_s)) return;
      }
    }
  }
};

static void test_mixed_simulation(int tp, uint64_t g0, int calls, unsigned seed,
                                  double timeout_s = 20.0) {
  MixedSim sim(tp, 40, calls, g0, seed);
  std::vector<std::thread> th;
  for (int r = 0; r < tp; ++r)
    th.emplace_back([&sim, r, seed, timeout_s] { sim.run_rank(r, seed * 17 + r, timeout_s); });
  for (auto& t : th) t.join();
  CHECK(sim.timeouts.load() == 0, "mixed tp %d: %d unexpected timeouts", tp, sim.timeouts.load());
  CHECK(sim.errors.load() == 0, "mixed tp %d: %d wrong sums", tp, sim.errors.load());
  std::printf("PASS mixed forward/backward simulation tp=%d g0=%llu calls=%d\n", tp,
              (unsigned long long)g0, calls);
}

static void test_simulation(int tp, uint64_t g0, int calls, unsigned seed) {
  Sim sim(tp, 48, calls, g0, seed);
  std::vector<std::thread> th;
  for (int r = 0; r < tp; ++r) th.emplace_back([&sim, r, seed] { sim.run_rank(r, seed * 31 + r, -1, 20.0); });
  for (auto& t : th) t.join();
  CHECK(sim.timeouts.load() == 0, "tp %d: %d unexpected timeouts", tp, sim.timeouts.load());
  CHECK(sim.errors.load() == 0, "tp %d: %d wrong sums", tp, sim.errors.load());
  std::printf("PASS simulation tp=%d g0=%llu calls=%d\n", tp, (unsigned long long)g0, calls);
}

static void test_skipped_call_times_out() {
  const int tp = 3, calls = 40, skip = 17;
  Sim sim(tp, 16, calls, (1ull << 32) - 20ull, 7);
  std::vector<std::thread> th;
  for (int r = 0; r < tp; ++r)
    th.emplace_back([&sim, r] { sim.run_rank(r, 100 + r, r == 1 ? skip : -1, 0.2); });
  for (auto& t : th) t.join();
  CHECK(sim.timeouts.load() >= 1, "a skipped call must make some wait run out");
  // The skipping rank goes from call skip-1 straight to skip+1, which uses the
  // same buffer as skip-1: its pushes may overwrite slots that slower peers
  // still await for skip-1. So the failure can surface one call early -- but
  // only ever as a bounded wait that runs out, never as a wrong sum.
  CHECK(sim.first_timeout_call.load() >= skip - 1, "timeout long before the skipped call (%lld)",
        sim.first_timeout_call.load());
  CHECK(sim.errors.load() == 0, "wrong sums before the skipped call");
  std::printf("PASS skipped call times out at call %lld\n", sim.first_timeout_call.load());
}

int main() {
#ifdef RTP_PLANT_EARLY_SECOND_PUSH
  test_mixed_simulation(4, 0ull, 2000, 5, 0.5);
  std::printf("%d FAILURES\n", g_failures);
  return g_failures ? 1 : 0;
#endif
  test_generation();
  test_packing();
  const uint64_t P = 0xFFFFFFFFull;
  test_simulation(2, 0ull, 3000, 1);
  test_simulation(4, P - 1500ull, 3000, 2);           // crosses the tag period
  test_simulation(8, (1ull << 32) - 1000ull, 2000, 3); // crosses the 32-bit wrap
  test_skipped_call_times_out();
  test_mixed_simulation(2, 0ull, 3000, 4);
  test_mixed_simulation(4, P - 1500ull, 2000, 5);           // crosses the tag period
  test_mixed_simulation(8, (1ull << 32) - 1000ull, 1500, 6); // crosses the 32-bit wrap
  if (g_failures) {
    std::printf("%d FAILURES\n", g_failures);
    return 1;
  }
  std::printf("ALL PASS\n");
  return 0;
}
