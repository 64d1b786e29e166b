// Producer side of the row-unit scheduling of the streaming kernels
// (scan_fwd.cu, scan_bwd.cu); the policy and the counter protocol are
// described with UnitSched in internal.h.
//
// One thread (thread 0) issues every chunk copy of its CTA.  Its state lives
// in shared memory, so it costs the other threads no registers, except the
// pending counter claim: that stays in a register so the atomic's latency
// is only paid where the value is used, one unit later.
#pragma once

#include "claim.h"
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

// The claim protocol (claim.h) on CUDA atomics.
struct DeviceAtomics {
  __device__ __forceinline__ unsigned add(unsigned* p) { return atomicAdd(p, 1u); }
  __device__ __forceinline__ void reset(unsigned* p) { atomicExch(p, 0u); }
};

// CTA b starts with unit b; with a counter it also claims its next unit.
template <int CH>
__device__ __forceinline__ void prod_init(ProdState& ps, const UnitSched& us, int64_t rows,
                                          int lg, unsigned& claim) {
  ps.unit = blockIdx.x;
  ps.k = 0;
  ps.issued = 0;
  ps.done = 0;
  prod_geom<CH>(ps, us, rows, lg);
  DeviceAtomics at;
  first_claim_t(us, claim, at);
}

// The unit claimed earlier (>= nunits: no more work); claims the next one.
__device__ __forceinline__ int64_t take_claim(const UnitSched& us, unsigned& claim) {
  DeviceAtomics at;
  return take_claim_t(us, claim, (int64_t)gridDim.x, at);
}

// Moves to the unit claimed earlier and claims the one after it.
template <int CH>
__device__ __forceinline__ void prod_next_unit(ProdState& ps, const UnitSched& us, int64_t rows,
                                               int lg, unsigned& claim) {
  ps.unit = take_claim(us, claim);
  if (ps.unit < us.nunits) prod_geom<CH>(ps, us, rows, lg);
}

// After an abort: the CTA's remaining claims (claim.h, drain_claims_t).
__device__ __forceinline__ void drain_claims(int64_t unit, const UnitSched& us, unsigned& claim) {
  DeviceAtomics at;
  drain_claims_t(unit, us, claim, (int64_t)gridDim.x, at);
}

}  // namespace fpscan
