// Internal launcher interface between the C-ABI layer (capi.cu) and the
// kernel translation units.  Not part of the public ABI.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace fpscan {

enum DType : int { kF32 = 0, kF16 = 1, kBF16 = 2 };

inline int dtype_size(int dt) { return dt == kF32 ? 4 : 2; }

inline int ilog2_host(int64_t v) {
  int r = 0;
  while ((int64_t(1) << (r + 1)) <= v) ++r;
  return r;
}

// Chained sequence sharding: per-row hand-off between neighbouring ranks
// through peer-mapped memory (see fpscan_link_* in capi.cu for the layout).
// in_word: values arriving from the upstream rank (local memory; 64-bit
// words epoch << 32 | float bits); ack_out: the upstream rank's ack word per
// row (peer memory), set to the epoch once the value is taken.  out_word:
// the downstream rank's slot (peer memory); ack_in: this rank's ack words,
// written by the downstream rank.  A row's out word is written only after
// ack_in shows the slot's previous use (epoch - depth) taken.
struct LinkParams {
  const uint64_t* in_word = nullptr;
  uint32_t* ack_out = nullptr;
  uint64_t* out_word = nullptr;
  const uint32_t* ack_in = nullptr;
  float* in_record = nullptr;  // optional: received values are also stored here
  uint32_t epoch = 0;
  uint32_t depth = 1;
};

// Row-unit scheduling of the streaming kernels (scan_fwd.cu, scan_bwd.cu).
// Streaming kernels cut their rows into units of `upr` whole rows.  Statically
// tiled, a one-wave grid finishes when its slowest CTA does, and CTAs of one
// launch were measured to finish up to 2x apart on B200 (a plain 2-read /
// 1-write stream: first CTA done at 625 us of 1283 us).  So CTA b takes unit b
// first and then claims further units from a 32-bit counter in global memory
// (one atomicAdd per unit, issued one unit ahead so its latency is hidden).
// Each launch makes exactly `nunits` claims: one per unit beyond the first
// wave plus one failing claim per CTA.  The claim that returns nunits - 1 is
// therefore the launch's last atomic on the counter, and its owner resets
// the word to 0 for the next launch on the same counter.  The host gives
// concurrent launches different counters (capi.cu, sched_counter).
struct UnitSched {
  unsigned* ctr = nullptr;  // null: static tiling, unit b = CTA b's whole tile
  int64_t upr = 1;                    // rows per unit
  int64_t nunits = 0;
  int64_t grid = 0;                   // CTAs to launch
};

// Units of at least kUnitChunks chunks (and whole rows); static tiling (one
// unit of ceil(rows / slots) rows per CTA) when there is no counter or fewer
// than two units per resident CTA: claiming balances CTAs of unequal speed
// only when each takes several units, while a second wave of a few large
// units would run alone (512 rows of 100000 on 444 slots: 3.7 TB/s claimed,
// 5.0 TB/s as 256 static tiles of 2 rows).
constexpr int64_t kUnitChunks = 4;
inline UnitSched plan_units(int64_t rows, int64_t seqlen, int64_t chunk, int64_t slots,
                            unsigned* ctr) {
  UnitSched u;
  if (ctr != nullptr) {
    int64_t upr = kUnitChunks * chunk / seqlen;
    if (upr < 1) upr = 1;
    const int64_t nunits = (rows + upr - 1) / upr;
    if (nunits >= 2 * slots && nunits < (int64_t(1) << 31)) {
      u.ctr = ctr;
      u.upr = upr;
      u.nunits = nunits;
      u.grid = slots;
      return u;
    }
  }
  int64_t rpt = (rows + slots - 1) / slots;
  if (rpt < 1) rpt = 1;
  u.upr = rpt;
  u.nunits = (rows + rpt - 1) / rpt;
  u.grid = u.nunits;
  return u;
}

struct FwdArgs {
  const void* gates;
  const void* tokens;
  void* out;            // nullptr: reduce only (carry-out required)
  const float* init;    // nullptr: zero initial state (first gate ignored)
  float* carry_a;       // nullptr: no carry-out; else per-row product of gates
  float* carry_b;       //          and per-row final state
  int64_t rows;
  int64_t seqlen;
  int dtype;
  int reverse;
  int num_sms;
  cudaStream_t stream;
  int nv = 2;           // 16-byte vectors per thread per chunk (1 or 2)
  int act = 0;          // gate activation applied on load (Act); plain scan only
  int link = 0;         // bit 0: init from link.in_*; bit 1: final state to link.out_*
  LinkParams lk;
  unsigned* sched = nullptr;  // unit counter (dynamic scheduling); null: static tiles
};

struct BwdArgs {
  const void* gates;
  const void* y;         // forward output; unused in reduce mode
  const void* grad_out;
  void* dgates;          // nullptr together with dtokens: reduce mode
  void* dtokens;
  const float* addend;   // nullptr: zero; else per-row value added at the row's last element
  const float* y_prev;   // nullptr: zero; else per-row y just before the row's first element
  float* carry_b;        // reduce mode: per-row gates[first] * dtokens[first]
  int64_t rows;
  int64_t seqlen;
  int dtype;
  int num_sms;
  cudaStream_t stream;
  int nv = 2;           // 16-byte vectors per thread per chunk (1 or 2)
  int act = 0;          // gate activation (Act): dgates becomes d/dz; plain backward only
  int link = 0;         // bit 0: addend from link.in_*; bit 1: carry to link.out_*
  LinkParams lk;
  unsigned* sched = nullptr;  // unit counter (dynamic scheduling); null: static tiles
};

struct SplitArgs {
  const void* gates;
  const void* tokens;
  void* out;
  void* workspace;      // >= split_workspace_bytes(rows, segments), 16-byte aligned
  int64_t rows;
  int64_t seqlen;
  int64_t segments;     // per row, power of two (split_segments)
  int dtype;
  int reverse;
  cudaStream_t stream;
};

// Split-row fused backward (scan_split.cu).
struct SplitBwdArgs {
  const void* gates;
  const void* y;
  const void* grad_out;
  void* dgates;
  void* dtokens;
  void* workspace;      // >= split_workspace_bytes(rows, segments), 16-byte aligned
  int64_t rows;
  int64_t seqlen;
  int64_t segments;     // per row, power of two (split_bwd_segments)
  int dtype;
  cudaStream_t stream;
};

// Scan / backward for any seqlen >= 1 (scan_anylen.cu).
struct AnyArgs {
  const void* gates;
  const void* tokens;    // forward
  void* out;             // forward
  const void* y;         // backward: forward output
  const void* grad_out;  // backward
  void* dgates;          // backward
  void* dtokens;         // backward
  int64_t rows;
  int64_t seqlen;
  int dtype;
  int reverse;           // forward only
  int backward;
  int num_sms;
  cudaStream_t stream;
  int nv = 1;            // 16-byte vectors per thread per chunk (1 or 2)
};

// Channel-last (batch, seqlen, dim) scan / backward (scan_cl.cu).
struct ClArgs {
  const void* gates;
  const void* tokens;    // forward
  void* out;             // forward
  const void* y;         // backward
  const void* grad_out;  // backward
  void* dgates;          // backward
  void* dtokens;         // backward
  void* workspace;       // >= cl_workspace_bytes(), 16-byte aligned
  uint64_t workspace_bytes;
  int64_t batch;
  int64_t seqlen;
  int64_t dim;
  int dtype;
  int reverse;
  int backward;
  cudaStream_t stream;
};

// Launches `kern` on `stream` with programmatic stream serialization (the
// kernel calls pdl_wait() before its first global access), so its prologue
// overlaps the tail of the previous kernel in the stream.
// FPSCAN_B200_PDL=0 launches without the attribute.
bool pdl_enabled();
// Whether the chained (link) kernels claim row units dynamically like the
// other streaming kernels (default) instead of static row tiles;
// FPSCAN_B200_LINK_CLAIM=0 gives static tiles.
bool link_claims();
template <typename K, typename P>
cudaError_t launch_pdl(K kern, unsigned grid, unsigned threads, size_t smem, cudaStream_t stream,
                       const P& p) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

// Records `fmt` as this thread's fpscan_last_error() message; returns code.
int set_error(int code, const char* fmt, ...);

cudaError_t launch_fwd(const FwdArgs& a);
cudaError_t launch_split(const SplitArgs& a);
int split_slots(int dtype, int num_sms);
int split_segments(int64_t rows, int64_t seqlen, int dtype, int slots);
int64_t split_workspace_bytes(int64_t rows, int segments);
cudaError_t launch_bwd(const BwdArgs& a);
int split_bwd_segments(int64_t rows, int64_t seqlen, int dtype, int num_sms);
cudaError_t launch_split_bwd(const SplitBwdArgs& a);
cudaError_t launch_anylen(const AnyArgs& a);
cudaError_t launch_cl(const ClArgs& a);
int64_t cl_workspace_bytes(int64_t batch, int64_t seqlen, int64_t dim, int dtype, bool backward);
cudaError_t launch_carry_combine(const float* gathered, int world, int rank, int64_t rows,
                                 int reverse, float* out, cudaStream_t stream);

}  // namespace fpscan
