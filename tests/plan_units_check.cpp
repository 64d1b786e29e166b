// Host-side check of the row-unit planner (fpscan_b200/csrc/internal.h,
// plan_units), compiled and run by tests/test_host_cpu.py: static tiles
// without a counter or with fewer than two units per CTA slot, claimed units
// otherwise; every plan covers the rows exactly once and fits one wave.
#include <cstdio>
#include <cstdlib>

#include "internal.h"

using fpscan::plan_units;
using fpscan::UnitSched;

static int failures = 0;
#define CHECK(cond, ...)                  \
  do {                                    \
    if (!(cond)) {                        \
      std::printf("FAIL %s: ", #cond);    \
      std::printf(__VA_ARGS__);           \
      std::printf("\n");                  \
      ++failures;                         \
    }                                     \
  } while (0)

int main() {
  unsigned word = 0;
  const int64_t chunks[] = {1024, 2048, 4096};
  const int64_t slots_list[] = {148, 444, 592};
  const int64_t seqlens[] = {1, 7, 32, 512, 1000, 2048, 4096, 8191, 16384, 65536, 100000};
  const int64_t rows_list[] = {1, 5, 148, 512, 592, 1183, 1184, 4096, 10240, 81920, 327680};
  for (int64_t chunk : chunks)
    for (int64_t slots : slots_list)
      for (int64_t L : seqlens)
        for (int64_t rows : rows_list)
          for (int with_ctr = 0; with_ctr < 2; ++with_ctr) {
            unsigned* ctr = with_ctr ? &word : nullptr;
            const UnitSched u = plan_units(rows, L, chunk, slots, ctr);
            CHECK(u.upr >= 1, "upr %lld", (long long)u.upr);
            CHECK(u.nunits == (rows + u.upr - 1) / u.upr, "nunits %lld rows %lld upr %lld",
                  (long long)u.nunits, (long long)rows, (long long)u.upr);
            CHECK(u.grid >= 1 && u.grid <= slots, "grid %lld slots %lld", (long long)u.grid,
                  (long long)slots);
            if (u.ctr == nullptr) {
              // static: one unit per CTA, all rows covered, no empty CTA
              CHECK(u.grid == u.nunits, "static grid %lld nunits %lld", (long long)u.grid,
                    (long long)u.nunits);
              CHECK(u.upr == (rows + slots - 1) / slots || (rows < slots && u.upr == 1),
                    "static upr %lld rows %lld slots %lld", (long long)u.upr, (long long)rows,
                    (long long)slots);
              CHECK((u.grid - 1) * u.upr < rows, "empty static tile");
            } else {
              // claimed: a full wave, at least two units per CTA, units of
              // >= 4 chunks (or one row when a row is longer)
              CHECK(with_ctr, "counter without one");
              CHECK(u.grid == slots, "claimed grid %lld", (long long)u.grid);
              CHECK(u.nunits >= 2 * slots, "claimed with %lld units for %lld slots",
                    (long long)u.nunits, (long long)slots);
              CHECK(u.upr == (4 * chunk / L > 1 ? 4 * chunk / L : 1), "claimed upr %lld",
                    (long long)u.upr);
            }
            if (with_ctr) {
              // the counter is used exactly when there are enough units
              const int64_t upr_c = 4 * chunk / L > 1 ? 4 * chunk / L : 1;
              const int64_t nu = (rows + upr_c - 1) / upr_c;
              CHECK((u.ctr != nullptr) == (nu >= 2 * slots), "choice rows %lld L %lld",
                    (long long)rows, (long long)L);
            }
          }
  std::printf(failures ? "%d failures\n" : "ok\n", failures);
  return failures ? 1 : 0;
}
