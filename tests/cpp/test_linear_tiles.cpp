// Host check of the fused linear's tile order (rmsnorm_tp_b200/csrc/rtp_common.h
// linear_tile): every (m block, n block) of the output is produced exactly once,
// and consecutive tiles of a group go to different owners (tp > 1).
#include <cstdio>
#include <vector>

#include "rtp_common.h"

int main() {
  int fails = 0;
  const int tps[] = {1, 2, 3, 4, 8};
  const long mts[] = {1, 2, 15, 16, 17, 33, 64};
  const long nbls[] = {1, 2, 4, 8};
  for (int tp : tps)
    for (long mt : mts)
      for (long nbl : nbls) {
        const long nt = tp * nbl;
        std::vector<int> seen(mt * nt, 0);
        long prev_owner = -1, same_owner_runs = 0;
        for (long t = 0; t < mt * nt; ++t) {
          int64_t mb = -1, nb = -1;
          rtp::linear_tile(t, mt, nt, tp, nbl, &mb, &nb);
          if (mb < 0 || mb >= mt || nb < 0 || nb >= nt) {
            std::printf("FAIL out of range tp=%d mt=%ld nbl=%ld t=%ld -> (%ld, %ld)\n", tp, mt, nbl,
                        t, (long)mb, (long)nb);
            ++fails;
            continue;
          }
          seen[mb * nt + nb] += 1;
          const long owner = nb / nbl;
          if (tp > 1 && t % 16 == 0 && t > 0 && owner == prev_owner) ++same_owner_runs;
          prev_owner = owner;
        }
        for (long i = 0; i < mt * nt; ++i)
          if (seen[i] != 1) {
            std::printf("FAIL tile (%ld, %ld) produced %d times (tp=%d mt=%ld nbl=%ld)\n", i / nt,
                        i % nt, seen[i], tp, mt, nbl);
            ++fails;
            break;
          }
      }
  std::printf(fails ? "FAILED\n" : "ALL PASS\n");
  return fails ? 1 : 0;
}
