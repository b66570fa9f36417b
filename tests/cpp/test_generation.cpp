// Host test of the device generation counter, built from the same header the
// CUDA kernels use (rmsnorm_tp_b200/csrc/rtp_common.h: gen_share, gen_of).
//
// The counter holds kGenUnit x (generation of the next launch), plus the shares
// the CTAs of a running one-generation launch have added. Every CTA reads it
// once (the launch's generation is the read >> kGenShift) and only afterwards
// advances it, as finish_launch (device_common.cuh) does: a one-generation
// launch by its share (gen_share: CTA 0 kGenUnit - (grid - 1), the others 1), a
// two-generation launch (backward) by the store of its last CTA, found by a
// returning add on the `done` count. The next launch reads it only after the
// whole grid has finished.
//
// Threads play the CTAs of many launches: grids of 1 to 4096 CTAs, one- and
// two-generation launches mixed, CTAs in random order with random delays
// between a CTA's read and its advance, so that reads meet every partial sum of
// the shares. Every CTA must read its launch's generation, and every finished
// launch must leave the counter at exactly kGenUnit x (generation + step) --
// from generation 0, just below the 32-bit tag wrap and just below the
// counter's largest generation. Built with -DRTP_PLANT_ADD_BEFORE_READ, a CTA
// advances the counter before it reads it (a planted mistake): the last CTA of
// every launch then reads the next generation, and the program must report
// failures.
#include <algorithm>
#include <atomic>
#include <cstdio>
#include <random>
#include <thread>
#include <vector>

#include "rtp_common.h"

using namespace rtp;

static std::atomic<int> g_failures{0};
#define CHECK(cond, ...)                                 \
  do {                                                   \
    if (!(cond)) {                                       \
      if (g_failures.fetch_add(1) < 10) {                \
        std::printf("FAIL %s:%d: ", __FILE__, __LINE__); \
        std::printf(__VA_ARGS__);                        \
        std::printf("\n");                               \
      }                                                  \
    }                                                    \
  } while (0)

// finish_launch's advance for one CTA
static void advance(std::atomic<uint64_t>& counter, std::atomic<uint32_t>& done, uint32_t cta,
                    uint32_t grid, uint64_t step, uint64_t g) {
  if (step == 1) {
    counter.fetch_add(gen_share(cta, grid), std::memory_order_relaxed);
  } else if (done.fetch_add(1u) == grid - 1u) {
    done.store(0u);
    counter.store((g + step) << kGenShift, std::memory_order_relaxed);
  }
}

// One launch of `grid` CTAs played by `workers` threads in a random order.
static void run_launch(std::atomic<uint64_t>& counter, std::atomic<uint32_t>& done, uint32_t grid,
                       uint64_t step, uint64_t expected, int workers, unsigned seed) {
  std::vector<uint32_t> order(grid);
  for (uint32_t i = 0; i < grid; ++i) order[i] = i;
  std::mt19937 rng(seed);
  std::shuffle(order.begin(), order.end(), rng);
  std::atomic<uint32_t> next{0};
  std::vector<std::thread> pool;
  for (int w = 0; w < workers; ++w) {
    pool.emplace_back([&, w] {
      std::mt19937 r(seed * 131u + (unsigned)w);
      for (;;) {
        const uint32_t k = next.fetch_add(1);
        if (k >= grid) break;
        const uint32_t cta = order[k];
#ifdef RTP_PLANT_ADD_BEFORE_READ
        advance(counter, done, cta, grid, step, expected);
        const uint64_t g = gen_of(counter.load(std::memory_order_relaxed));
#else
        const uint64_t g = gen_of(counter.load(std::memory_order_relaxed));
        for (unsigned spin = r() % 64u; spin > 0; --spin) std::this_thread::yield();
        advance(counter, done, cta, grid, step, g);
#endif
        CHECK(g == expected, "launch of %u CTAs, generation %llu: CTA %u read %llu", grid,
              (unsigned long long)expected, cta, (unsigned long long)g);
      }
    });
  }
  for (auto& t : pool) t.join();   // the grid has finished
}

int main() {
  // the shares of any grid add up to one unit, and the shares of all CTAs but
  // any one stay below it (with CTA 0's: kGenUnit - 1 at most; without: grid - 1)
  for (uint32_t grid : {1u, 2u, 3u, 148u, 296u, 4096u, (uint32_t)(kGenUnit / 2)}) {
    uint64_t total = 0;
    for (uint32_t c = 0; c < grid; ++c) total += gen_share(c, grid);
    CHECK(total == kGenUnit, "grid %u: shares sum to %llu", grid, (unsigned long long)total);
    for (uint32_t left_out : {0u, grid - 1u}) {
      const uint64_t rest = total - gen_share(left_out, grid);
      CHECK(grid == 1u || rest < kGenUnit, "grid %u: all but CTA %u reach a unit", grid, left_out);
    }
  }

  const int workers = (int)std::max(4u, std::thread::hardware_concurrency());
  const uint64_t starts[] = {0ull, 0xFFFFFFFFull - 40ull, kGenMax - 400ull};
  std::mt19937 rng(12345);
  for (uint64_t g0 : starts) {
    std::atomic<uint64_t> counter{g0 << kGenShift};
    std::atomic<uint32_t> done{0u};
    uint64_t g = g0;
    for (int launch = 0; launch < 120; ++launch) {
      const uint32_t grid = 1u + rng() % (launch % 3 == 0 ? 4096u : 300u);
      const uint64_t step = (rng() % 3u == 0u) ? 2ull : 1ull;
      run_launch(counter, done, grid, step, g, workers, (unsigned)rng());
      g += step;
      CHECK(counter.load() == (g << kGenShift), "after launch %d: counter %llu, want %llu",
            launch, (unsigned long long)counter.load(), (unsigned long long)(g << kGenShift));
    }
  }
  if (g_failures.load() == 0) {
    std::printf("ALL PASS\n");
    return 0;
  }
  std::printf("%d failures\n", g_failures.load());
  return 1;
}
