// Counter protocol of the row-unit claiming (UnitSched, internal.h), written
// once for the kernels (CUDA atomics, sched.cuh) and for the host-side test
// that runs it with CPU threads as CTAs (tests/claim_protocol_check.cpp).
//
// `Atomics` provides add(p): atomically p += 1, returning the old value, and
// reset(p): atomically p = 0.
#pragma once

#include <cstdint>

#include "internal.h"

#if defined(__CUDACC__)
#define FPSCAN_CLAIM_FN __device__ __forceinline__
#else
#define FPSCAN_CLAIM_FN inline
#endif

namespace fpscan {

// First claim of a CTA (which starts with unit = its index): the unit after it.
template <class Atomics>
FPSCAN_CLAIM_FN void first_claim_t(const UnitSched& us, unsigned& claim, Atomics& at) {
  if (us.ctr != nullptr) claim = at.add(us.ctr);
}

// Consumes the pending claim: returns the unit claimed earlier (>= nunits:
// no more work) and, if it is one, claims the unit after it.  The launch's
// last claim (value nunits - 1) resets the counter.  Static tiling (no
// counter): no unit after the first.
template <class Atomics>
FPSCAN_CLAIM_FN int64_t take_claim_t(const UnitSched& us, unsigned& claim, int64_t grid,
                                     Atomics& at) {
  if (us.ctr == nullptr) return us.nunits;
  if ((int64_t)claim == us.nunits - 1) at.reset(us.ctr);
  const int64_t u = grid + (int64_t)claim;
  if (u < us.nunits) claim = at.add(us.ctr);
  return u;
}

// After an abort: makes the CTA's remaining claims (its failing one
// included), so the counter is still reset by the launch's last claim.
template <class Atomics>
FPSCAN_CLAIM_FN void drain_claims_t(int64_t unit, const UnitSched& us, unsigned& claim,
                                    int64_t grid, Atomics& at) {
  while (us.ctr != nullptr && unit < us.nunits) unit = take_claim_t(us, claim, grid, at);
}

}  // namespace fpscan
