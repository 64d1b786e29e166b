// Host-side check of the row-unit claim protocol (fpscan_b200/csrc/claim.h),
// compiled and run by tests/test_host_cpu.py.  Each simulated launch runs one
// thread per CTA on a shared counter word, as the kernels' producer thread
// does: CTA b takes unit b, claims its next unit ahead, and consumes the
// claim when it moves on.  Checks, over many launches that reuse one word:
// every unit is processed exactly once, and the word is 0 after the launch
// (so the next launch starts clean) -- also when CTAs abort and drain.
#include <atomic>
#include <cstdio>
#include <random>
#include <thread>
#include <vector>

#include "claim.h"

using fpscan::UnitSched;

struct HostAtomics {
  unsigned add(unsigned* p) { return __atomic_fetch_add(p, 1u, __ATOMIC_SEQ_CST); }
  void reset(unsigned* p) { __atomic_store_n(p, 0u, __ATOMIC_SEQ_CST); }
};

static int failures = 0;

// One launch of `grid` CTAs over `nunits` units.  CTAs listed in `abort_at`
// stop after that many units and drain their claims.
static void launch(unsigned* word, int64_t grid, int64_t nunits, unsigned seed,
                   const std::vector<int>& abort_after) {
  UnitSched us;
  us.ctr = word;
  us.upr = 1;
  us.nunits = nunits;
  us.grid = grid;
  std::vector<std::atomic<int>> done(nunits);
  for (auto& d : done) d = 0;
  std::vector<int> aborted_units(grid, 0);
  std::vector<std::thread> ctas;
  for (int64_t b = 0; b < grid; ++b) {
    ctas.emplace_back([&, b] {
      std::mt19937 rng(seed * 7919u + (unsigned)b);
      HostAtomics at;
      unsigned claim = 0;
      int64_t unit = b;
      fpscan::first_claim_t(us, claim, at);
      int processed = 0;
      while (unit < us.nunits) {
        if (abort_after[b] >= 0 && processed == abort_after[b]) {
          // abort: the current unit is not processed; claims are drained
          fpscan::drain_claims_t(unit, us, claim, grid, at);
          aborted_units[b] = 1;
          return;
        }
        done[unit].fetch_add(1);
        ++processed;
        for (unsigned y = rng() % 3; y > 0; --y) std::this_thread::yield();
        unit = fpscan::take_claim_t(us, claim, grid, at);
      }
    });
  }
  for (auto& t : ctas) t.join();
  bool any_abort = false;
  for (int v : aborted_units) any_abort |= v != 0;
  int64_t twice = 0, missing = 0;
  for (auto& d : done) {
    if (d > 1) ++twice;
    if (d == 0) ++missing;
  }
  if (twice) {
    std::printf("FAIL grid %lld units %lld: %lld units processed twice\n", (long long)grid,
                (long long)nunits, (long long)twice);
    ++failures;
  }
  if (missing && !any_abort) {
    std::printf("FAIL grid %lld units %lld: %lld units never processed\n", (long long)grid,
                (long long)nunits, (long long)missing);
    ++failures;
  }
  const unsigned left = __atomic_load_n(word, __ATOMIC_SEQ_CST);
  if (left != 0) {
    std::printf("FAIL grid %lld units %lld: counter left at %u\n", (long long)grid,
                (long long)nunits, left);
    ++failures;
  }
}

int main() {
  unsigned word = 0;  // reused by every launch, as a graph replay reuses its word
  unsigned seed = 1;
  const int64_t grids[] = {1, 2, 7, 32, 148};
  for (int rep = 0; rep < 2; ++rep)
    for (int64_t grid : grids)
      for (int64_t mult : {1, 3, 17}) {
        const int64_t nunits = grid * mult + (mult > 1 ? grid / 3 : 0);
        std::vector<int> none(grid, -1);
        launch(&word, grid, nunits, seed++, none);
        // some CTAs abort after 0, 1 or 2 units
        std::vector<int> some(grid, -1);
        for (int64_t b = 0; b < grid; b += 3) some[b] = (int)(b % 3);
        launch(&word, grid, nunits, seed++, some);
      }
  // the static plan (no counter) makes no claims
  {
    UnitSched us;
    us.nunits = 5;
    HostAtomics at;
    unsigned claim = 123;
    fpscan::first_claim_t(us, claim, at);
    if (claim != 123 || fpscan::take_claim_t(us, claim, 5, at) != 5) {
      std::printf("FAIL static plan claimed\n");
      ++failures;
    }
  }
  std::printf(failures ? "%d failures\n" : "ok\n", failures);
  return failures ? 1 : 0;
}
