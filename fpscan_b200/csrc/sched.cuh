// Producer side of the row-unit scheduling of the streaming kernels
// (scan_fwd.cu, scan_bwd.cu); the policy and the counter protocol are
// described with UnitSched in internal.h.
//
// One thread (thread 0) issues every chunk copy of its CTA.  Its state lives
// in shared memory, so it costs the other threads no registers, except the
// pending counter claim: that stays in a register so the atomic's latency
// is only paid where the value is used, one unit later.
#pragma once

#include "common.cuh"
#include "internal.h"

namespace fpscan {

struct ProdState {
  int64_t unit;    // unit being issued (>= nunits: no more work)
  int64_t k;       // next chunk of the unit, in processing order
  int64_t base;    // the unit's first element
  int64_t n;       // its elements
  int64_t nck;     // its chunks
  int64_t issued;  // stage fills so far (chunks and the end marker)
  int done;        // end marker issued
};

template <int CH>
__device__ __forceinline__ void prod_geom(ProdState& ps, const UnitSched& us, int64_t rows,
                                          int lg) {
  const int64_t row0 = ps.unit * us.upr;
  ps.base = row0 << lg;
  ps.n = min(us.upr, rows - row0) << lg;
  ps.nck = (ps.n + CH - 1) / CH;
}

// CTA b starts with unit b; with a counter it also claims its next unit.
template <int CH>
__device__ __forceinline__ void prod_init(ProdState& ps, const UnitSched& us, int64_t rows,
                                          int lg, unsigned& claim) {
  ps.unit = blockIdx.x;
  ps.k = 0;
  ps.issued = 0;
  ps.done = 0;
  prod_geom<CH>(ps, us, rows, lg);
  if (us.ctr != nullptr) claim = atomicAdd(us.ctr, 1u);
}

// Consumes the pending claim: returns the unit claimed earlier (>= nunits:
// no more work) and, if it is one, claims the unit after it.  The launch's
// last claim (value nunits - 1) resets the counter.  Static tiling (no
// counter): no unit after the first.
__device__ __forceinline__ int64_t take_claim(const UnitSched& us, unsigned& claim) {
  if (us.ctr == nullptr) return us.nunits;
  if ((int64_t)claim == us.nunits - 1) atomicExch(us.ctr, 0u);
  const int64_t u = (int64_t)gridDim.x + (int64_t)claim;
  if (u < us.nunits) claim = atomicAdd(us.ctr, 1u);
  return u;
}

// Moves to the unit claimed earlier and claims the one after it.
template <int CH>
__device__ __forceinline__ void prod_next_unit(ProdState& ps, const UnitSched& us, int64_t rows,
                                               int lg, unsigned& claim) {
  ps.unit = take_claim(us, claim);
  if (ps.unit < us.nunits) prod_geom<CH>(ps, us, rows, lg);
}

// After an abort: makes the CTA's remaining claims (its failing one
// included), so the counter is still reset by the launch's last claim.
__device__ __forceinline__ void drain_claims(int64_t unit, const UnitSched& us, unsigned& claim) {
  while (us.ctr != nullptr && unit < us.nunits) unit = take_claim(us, claim);
}

}  // namespace fpscan
