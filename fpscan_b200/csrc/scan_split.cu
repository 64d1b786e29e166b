// Split-row forward / reverse scan for few, long rows, sm_100a.
//
// When batch*dim is far smaller than the number of CTA slots of the GPU,
// one CTA per row leaves SMs idle and keeps too few bytes in flight.  Here every row is cut into segments of 4 chunks
// (32 KiB per tensor) and each segment is one tile, taken in order from an
// atomic tile counter (so every tile's predecessors are already running):
//   stage   the whole segment (gates and tokens, 64 KiB) with non-multicast
//           bulk copies issued at once, one mbarrier per chunk;
//   pass A  composes the segment's affine map (A, B) chunk by chunk as the
//           copies land;
//   publish the map (flag AGG) -- or, for a row's first segment, its final
//           state (flag INCL);
//   look back over the preceding segments of the row (decoupled look-back:
//           combine AGG maps until an INCL state is found), publish INCL;
//   pass B  rescans the staged chunks with the carried-in state, writes y.
// DRAM traffic is exactly 2 reads + 1 write per element.
//
// Scratch (caller's workspace, fpscan_scan_fwd_workspace_bytes):
//   [0, 8)    tile counter, zeroed by an async memset before every launch;
//   [256, ..) one 16-byte status word per tile {A, B, B_incl, flag}.  Flags carry
//             a per-launch epoch, so stale words from earlier launches are
//             never mistaken for this launch's and need no clearing.
// Look-back spins are bounded (g_wait_limit_ns, 2 s by default); on timeout
// the tile uses state NaN (its row comes out visibly wrong) and the device
// status word records kStatusLookbackTimeout.
#include "common.cuh"
#include "internal.h"

#include <atomic>

namespace fpscan {

struct __align__(16) SegStatus {
  float a;       // segment map (published with the AGG flag, never rewritten)
  float b;
  float b_incl;  // state at the segment's end (published with the INCL flag)
  uint32_t flag;  // (epoch << 1) | is_inclusive
};

struct SplitKParams {
  const void* gates;
  const void* tokens;
  void* out;
  unsigned long long* counter;
  SegStatus* status;
  int64_t rows;
  int lg;      // log2(seqlen)
  int lgp;     // log2(segments per row)
  uint32_t epoch;
};

constexpr int kSplitNV = 2;
constexpr int kSegChunks = 4;  // a segment = 4 chunks, staged whole in shared memory
constexpr int kSplitSmem = kSegChunks * 2 * kThreads * kSplitNV * 16;

__device__ __forceinline__ void st_release(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Thread 0 of tile t (processing-order segment sp of its row): publishes the
// segment's map (agg_a, agg_b), looks back over the row's preceding
// segments (combining aggregate maps until an inclusive state is found),
// publishes the segment's inclusive state and returns the state entering
// the segment.  A row's first segment starts from the zero state (its map's
// B is its final state).  Spins are bounded by g_wait_limit_ns; on timeout
// the state is NaN and kStatusLookbackTimeout is recorded.
__device__ float split_publish_lookback(SegStatus* status, int64_t t, int64_t sp, float agg_a,
                                        float agg_b, uint32_t epoch) {
  SegStatus* st = status + t;
  const uint32_t agg_flag = epoch << 1, incl_flag = (epoch << 1) | 1u;
  if (sp == 0) {
    st->b_incl = agg_b;
    st_release(&st->flag, incl_flag);
    return 0.f;
  }
  st->a = agg_a;
  st->b = agg_b;
  st_release(&st->flag, agg_flag);
  float state_in = 0.f;
  float acc_a = 1.f, acc_b = 0.f;  // composition of the segments after j, before t
  const uint64_t t0 = global_ns();
  for (int64_t j = t - 1;; --j) {
    const SegStatus* sj = status + j;
    uint32_t f;
    uint32_t spins = 0;
    bool timed_out = false;
    while (true) {
      f = ld_acquire(&sj->flag);
      if ((f >> 1) == epoch) break;
      if ((++spins & 63u) == 0 &&
          global_ns() - t0 > *(volatile unsigned long long*)&g_wait_limit_ns) {
        timed_out = true;
        break;
      }
    }
    if (timed_out) {
      atomicOr(&g_status, kStatusLookbackTimeout);
      state_in = __int_as_float(0x7fc00000);  // NaN: the row is visibly wrong
      break;
    }
    if (f & 1u) {
      state_in = fmaf(__ldcg(&sj->b_incl), acc_a, acc_b);
      break;
    }
    const float ja = __ldcg(&sj->a), jb = __ldcg(&sj->b);
    acc_b = fmaf(jb, acc_a, acc_b);
    acc_a *= ja;
  }
  st->b_incl = fmaf(agg_a, state_in, agg_b);
  st_release(&st->flag, incl_flag);
  return state_in;
}

template <typename T, bool REV>
__global__ void __launch_bounds__(kThreads, 3) scan_split_kernel(const SplitKParams p) {
  constexpr int NV = kSplitNV;
  constexpr int V = Elem<T>::kVec;
  constexpr int E = V * NV;
  constexpr int CH = kThreads * E;
  constexpr int LGCH = ilog2(CH);
  constexpr int NC = kSegChunks;
  constexpr int SV = kThreads * NV;

  extern __shared__ __align__(128) uint4 dsm[];
  uint4 (*s_g)[SV] = reinterpret_cast<uint4 (*)[SV]>(dsm);            // [NC][SV]
  uint4 (*s_x)[SV] = reinterpret_cast<uint4 (*)[SV]>(dsm + NC * SV);  // [NC][SV]
  __shared__ __align__(8) uint64_t s_bar[NC];
  __shared__ float2 s_wt[2][kWarps];
  __shared__ long long s_tile;
  __shared__ float s_state;

  const T* __restrict__ gates = static_cast<const T*>(p.gates);
  const T* __restrict__ tokens = static_cast<const T*>(p.tokens);
  T* out = static_cast<T*>(p.out);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  pdl_wait();  // the previous kernel in the stream is complete from here on
  pdl_launch_dependents();
  if (tid == 0) {
    s_tile = (long long)atomicAdd(p.counter, 1ull);
#pragma unroll
    for (int c = 0; c < NC; ++c) mbar_init(&s_bar[c], 1);
    fence_mbar_init();
  }
  __syncthreads();
  const int64_t t = s_tile;
  const int64_t P = int64_t(1) << p.lgp;
  if (t >= (p.rows << p.lgp)) return;
  const int64_t row = t >> p.lgp;
  const int64_t sp = t & (P - 1);             // segment index in processing order
  const int64_t seg = REV ? P - 1 - sp : sp;  // segment index in memory order
  const int64_t base = (row << p.lg) + (seg << (LGCH + 2));  // NC == 4 chunks per segment

  FPSCAN_DEBUG_ONLY(const int64_t n_el = p.rows << p.lg;)  // elements of each tensor
  // Stage the whole segment at once: chunk c (processing order) -> buffer c.
  if (tid == 0) {
    const uint32_t bytes = (uint32_t)(CH * sizeof(T));
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int64_t off = (int64_t)(REV ? NC - 1 - c : c) << LGCH;
      // debug builds: a copy outside its tensor is skipped, the stage completes
      FPSCAN_DEBUG_ONLY(
          if (!in_bounds(gates + base + off, bytes, gates, gates + n_el) ||
              !in_bounds(tokens + base + off, bytes, tokens, tokens + n_el)) {
            mbar_arrive(&s_bar[c]);
            continue;
          })
      mbar_expect_tx(&s_bar[c], 2u * bytes);
      bulk_g2s(s_g[c], gates + base + off, bytes, &s_bar[c]);
      bulk_g2s(s_x[c], tokens + base + off, bytes, &s_bar[c]);
    }
  }

  const int vi = REV ? kThreads - 1 - tid : tid;
  auto load_scan = [&](int c, float (&a)[E], float (&b)[E]) {
    uint4 rg[NV], rx[NV];
    lds_vecs<NV>(&s_g[c][vi * NV], rg);
    lds_vecs<NV>(&s_x[c][vi * NV], rx);
    Vec16<T> gv[NV], xv[NV];
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      gv[k].raw = rg[k];
      xv[k].raw = rx[k];
    }
#pragma unroll
    for (int i = 0; i < E; ++i) {
      const int j = REV ? E - 1 - i : i;
      const float g = Elem<T>::load(gv[j / V].e[j % V]);
      const float x = Elem<T>::load(xv[j / V].e[j % V]);
      if (i == 0) {
        a[0] = g;
        b[0] = x;
      } else {
        a[i] = a[i - 1] * g;
        b[i] = fmaf(b[i - 1], g, x);
      }
    }
  };

  // ---- pass A: the segment's map (agg_a, agg_b), chunk by chunk as they land
  float agg_a = 1.f, agg_b = 0.f;
  bool ok_all = true;
  int q = 0;  // barrier count, selects the s_wt buffer
  for (int c = 0; c < NC; ++c, ++q) {
    const bool ok = mbar_wait_bounded(&s_bar[c], 0);
    float a[E], b[E];
    load_scan(c, a, b);
    float ta = a[E - 1], tb = b[E - 1];
    warp_scan_pair(ta, tb, lane, 32);
    if (lane == 31) s_wt[q & 1][warp] = make_float2(ta, tb);
    if (__syncthreads_or(!ok)) {
      ok_all = false;
      break;
    }
    float pa = 1.f, pb = 0.f, ca, cb;
    compose_warp_totals(s_wt[q & 1], lane, warp, kWarps, pa, pb, ca, cb);
    if (c == 0) {
      agg_a = ca;
      agg_b = cb;
    } else {
      agg_b = fmaf(agg_b, ca, cb);
      agg_a *= ca;
    }
  }
  if (!ok_all) {
    if (tid == 0)
      for (int c = 0; c < NC; ++c) mbar_wait_bounded(&s_bar[c], 0);
    return;
  }

  // ---- publish, look back, publish the inclusive state
  if (tid == 0) {
    const float state_in = split_publish_lookback(p.status, t, sp, agg_a, agg_b, p.epoch);
    s_state = state_in;
  }
  __syncthreads();
  float carry = s_state;

  // ---- pass B: rescan the staged chunks with the carried-in state, write y
  for (int c = 0; c < NC; ++c, ++q) {
    const int64_t off = (int64_t)(REV ? NC - 1 - c : c) << LGCH;
    float a[E], b[E];
    load_scan(c, a, b);
    float ta = a[E - 1], tb = b[E - 1], pa, pb;
    warp_exclusive(ta, tb, lane, 32, pa, pb);
    if (lane == 31) s_wt[q & 1][warp] = make_float2(ta, tb);
    __syncthreads();
    float ca, cb;
    compose_warp_totals(s_wt[q & 1], lane, warp, kWarps, pa, pb, ca, cb);
    const bool row_start = (sp == 0 && c == 0);
    const bool skip_state = row_start && tid == 0;  // ignore the row's first gate
    const float state = row_start ? pb : fmaf(pa, carry, pb);
    float f[E];
#pragma unroll
    for (int i = 0; i < E; ++i)
      f[REV ? E - 1 - i : i] = skip_state ? b[i] : fmaf(a[i], state, b[i]);
    uint4* dst = reinterpret_cast<uint4*>(out + base + off) + vi * NV;
    FPSCAN_DEBUG_ONLY(if (in_bounds(dst, NV * 16, out, out + n_el)))
#pragma unroll
    for (int k2 = 0; k2 < NV; ++k2) dst[k2] = pack_vec<T>(f + k2 * V);
    carry = row_start ? cb : fmaf(ca, carry, cb);
  }
}

// ---------------------------------------------------------------- fused backward
// Split-row fused backward for few, long rows: the backward of scan_bwd.cu
// (dtokens[t] = gates[t+1] * dtokens[t+1] + grad_out[t], dgates[t] =
// dtokens[t] * y[t-1]) with rows cut into segments of kSegChunks chunks,
// each one tile taken in order from a counter, processed from the row's
// end.  Per tile: the segment's gates (plus the vector after it), grad_out
// and y (plus the vector before it) are staged whole by bulk copies; pass A
// composes the segment's map on the dtokens state entering from the right
// (element t: A = gates[t+1], B = grad_out[t]); the decoupled look-back
// (split_publish_lookback) yields that state; pass B re-runs the recurrence
// from it and writes dtokens and dgates.  DRAM traffic: 3 reads + 2 writes
// per element (plus two 16-byte halos per segment).
struct SplitBwdKParams {
  const void* gates;
  const void* y;
  const void* gout;
  void* dgates;
  void* dtok;
  unsigned long long* counter;
  SegStatus* status;
  int64_t rows;
  int lg;   // log2(seqlen)
  int lgp;  // log2(segments per row)
  uint32_t epoch;
};

constexpr int kSplitBwdNV = 1;
constexpr int kSplitBwdSV = kThreads * kSplitBwdNV;  // 16-byte vectors per chunk
// gates + one vector after, grad_out, one vector before + y
constexpr int kSplitBwdSmem = 16 * (3 * kSegChunks * kSplitBwdSV + 2);

template <typename T>
__global__ void __launch_bounds__(kThreads, 4) scan_split_bwd_kernel(const SplitBwdKParams p) {
  constexpr int NV = kSplitBwdNV;
  constexpr int V = Elem<T>::kVec;
  constexpr int E = V * NV;
  constexpr int CH = kThreads * E;
  constexpr int NC = kSegChunks;
  constexpr int SV = kSplitBwdSV;
  constexpr int64_t SE = (int64_t)NC * CH;  // elements per segment

  extern __shared__ __align__(128) uint4 dsm[];
  uint4* s_g = dsm;                 // [NC*SV + 1]: the segment's gates, then the vector after
  uint4* s_go = s_g + NC * SV + 1;  // [NC*SV]
  uint4* s_y = s_go + NC * SV;      // [1 + NC*SV]: the vector before, then the segment's y
  __shared__ __align__(8) uint64_t s_bar[NC];
  __shared__ float2 s_wt[2][kWarps];
  __shared__ long long s_tile;
  __shared__ float s_state;

  const T* __restrict__ gates = static_cast<const T*>(p.gates);
  const T* __restrict__ y = static_cast<const T*>(p.y);
  const T* __restrict__ gout = static_cast<const T*>(p.gout);
  T* dgates = static_cast<T*>(p.dgates);
  T* dtok = static_cast<T*>(p.dtok);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  pdl_wait();  // the previous kernel in the stream is complete from here on
  pdl_launch_dependents();
  if (tid == 0) {
    s_tile = (long long)atomicAdd(p.counter, 1ull);
#pragma unroll
    for (int c = 0; c < NC; ++c) mbar_init(&s_bar[c], 1);
    fence_mbar_init();
  }
  __syncthreads();
  const int64_t t = s_tile;
  const int64_t P = int64_t(1) << p.lgp;
  if (t >= (p.rows << p.lgp)) return;
  const int64_t row = t >> p.lgp;
  const int64_t sp = t & (P - 1);  // processing order: segment 0 holds the row's end
  const int64_t seg = P - 1 - sp;  // memory order
  const int64_t base = (row << p.lg) + seg * SE;
  const bool row_end_seg = sp == 0;
  const bool row_start_seg = seg == 0;
  FPSCAN_DEBUG_ONLY(const int64_t n_el = p.rows << p.lg;)  // elements of each tensor

  // Stage everything at once: chunk c (processing order) is memory chunk
  // NC-1-c and completes on barrier c; the gates halo rides with chunk 0,
  // the y halo with chunk NC-1.
  if (tid == 0) {
    const uint32_t bytes = (uint32_t)(CH * sizeof(T));
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int mc = NC - 1 - c;
      const int64_t off = (int64_t)mc * CH;
      const bool gh = c == 0 && !row_end_seg;
      const bool yh = c == NC - 1 && !row_start_seg;
      // debug builds: a copy outside its tensor is skipped, the stage completes
      FPSCAN_DEBUG_ONLY(
          if (!in_bounds(gates + base + off, bytes + (gh ? 16u : 0u), gates, gates + n_el) ||
              !in_bounds(gout + base + off, bytes, gout, gout + n_el) ||
              !in_bounds(yh ? y + base - V : y + base + off, bytes + (yh ? 16u : 0u), y,
                         y + n_el)) {
            mbar_arrive(&s_bar[c]);
            continue;
          })
      mbar_expect_tx(&s_bar[c], 3u * bytes + (gh ? 16u : 0u) + (yh ? 16u : 0u));
      bulk_g2s(s_g + mc * SV, gates + base + off, bytes + (gh ? 16u : 0u), &s_bar[c]);
      bulk_g2s(s_go + mc * SV, gout + base + off, bytes, &s_bar[c]);
      if (yh)
        bulk_g2s(s_y, y + base - V, bytes + 16u, &s_bar[c]);
      else
        bulk_g2s(s_y + 1 + mc * SV, y + base + off, bytes, &s_bar[c]);
    }
  }

  const int vi = kThreads - 1 - tid;  // vector slot, reverse processing order
  // The thread's map over its group of memory chunk mc (element t: A =
  // gates[t+1], B = grad_out[t]), folded in processing order; g_next =
  // gates of the element after the group (1 at the row's end).
  auto load_group = [&](int mc, Vec16<T> (&gv)[NV], Vec16<T> (&gov)[NV], float& g_next) {
    const uint4* sg = s_g + mc * SV + vi * NV;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      gv[k].raw = sg[k];
      gov[k].raw = s_go[mc * SV + vi * NV + k];
    }
    const bool at_row_end = row_end_seg && mc == NC - 1 && vi == kThreads - 1;
    g_next = at_row_end ? 1.f : Elem<T>::load(reinterpret_cast<const T*>(sg + NV)[0]);
  };
  auto fold = [&](const Vec16<T> (&gv)[NV], const Vec16<T> (&gov)[NV], float g_next, float& ta,
                  float& tb) {
#pragma unroll
    for (int i = 0; i < E; ++i) {
      const int j = E - 1 - i;
      const float a = (j == E - 1) ? g_next : Elem<T>::load(gv[(j + 1) / V].e[(j + 1) % V]);
      const float x = Elem<T>::load(gov[j / V].e[j % V]);
      if (i == 0) {
        ta = a;
        tb = x;
      } else {
        tb = fmaf(tb, a, x);
        ta *= a;
      }
    }
  };

  // ---- pass A: the segment's map, chunk by chunk as the copies land
  float agg_a = 1.f, agg_b = 0.f;
  bool ok_all = true;
  int q = 0;
  for (int c = 0; c < NC; ++c, ++q) {
    const bool ok = mbar_wait_bounded(&s_bar[c], 0);
    Vec16<T> gv[NV], gov[NV];
    float g_next, ta, tb;
    load_group(NC - 1 - c, gv, gov, g_next);
    fold(gv, gov, g_next, ta, tb);
    warp_scan_pair(ta, tb, lane, 32);
    if (lane == 31) s_wt[q & 1][warp] = make_float2(ta, tb);
    if (__syncthreads_or(!ok)) {
      ok_all = false;
      break;
    }
    float pa = 1.f, pb = 0.f, ca, cb;
    compose_warp_totals(s_wt[q & 1], lane, warp, kWarps, pa, pb, ca, cb);
    if (c == 0) {
      agg_a = ca;
      agg_b = cb;
    } else {
      agg_b = fmaf(agg_b, ca, cb);
      agg_a *= ca;
    }
  }
  if (!ok_all) {
    if (tid == 0)
      for (int c = 0; c < NC; ++c) mbar_wait_bounded(&s_bar[c], 0);
    return;
  }

  // ---- publish, look back, publish the inclusive state
  if (tid == 0) s_state = split_publish_lookback(p.status, t, sp, agg_a, agg_b, p.epoch);
  __syncthreads();
  float carry = s_state;

  // ---- pass B: the recurrence from the entering state; dtokens and dgates
  for (int c = 0; c < NC; ++c, ++q) {
    const int mc = NC - 1 - c;
    Vec16<T> gv[NV], gov[NV];
    float g_next, ta, tb, pa, pb;
    load_group(mc, gv, gov, g_next);
    fold(gv, gov, g_next, ta, tb);
    warp_exclusive(ta, tb, lane, 32, pa, pb);
    if (lane == 31) s_wt[q & 1][warp] = make_float2(ta, tb);
    __syncthreads();
    float ca, cb;
    compose_warp_totals(s_wt[q & 1], lane, warp, kWarps, pa, pb, ca, cb);
    const bool row_start = row_end_seg && c == 0;  // processing order: the row's end
    const float state = row_start ? pb : fmaf(pa, carry, pb);
    // y of the element before each one; before the group's first: the last
    // element of the previous vector (the halo for the segment's first
    // vector), 0 before the row's first element
    Vec16<T> yv[NV];
    const uint4* sy = s_y + 1 + mc * SV + vi * NV;
#pragma unroll
    for (int k = 0; k < NV; ++k) yv[k].raw = sy[k];
    const bool at_row_start = row_start_seg && mc == 0 && vi == 0;
    const float y_before = at_row_start ? 0.f : Elem<T>::load(reinterpret_cast<const T*>(sy)[-1]);
    float f_dt[E], f_dg[E];
    float d = state;
#pragma unroll
    for (int i = 0; i < E; ++i) {
      const int j = E - 1 - i;
      const float a = (j == E - 1) ? g_next : Elem<T>::load(gv[(j + 1) / V].e[(j + 1) % V]);
      d = fmaf(a, d, Elem<T>::load(gov[j / V].e[j % V]));
      const float yp = (j == 0) ? y_before : Elem<T>::load(yv[(j - 1) / V].e[(j - 1) % V]);
      f_dt[j] = d;
      f_dg[j] = d * yp;
    }
    const int64_t o = base + (int64_t)mc * CH;
    uint4* d1 = reinterpret_cast<uint4*>(dtok + o) + vi * NV;
    uint4* d2 = reinterpret_cast<uint4*>(dgates + o) + vi * NV;
    FPSCAN_DEBUG_ONLY(if (in_bounds(d1, NV * 16, dtok, dtok + n_el) &&
                          in_bounds(d2, NV * 16, dgates, dgates + n_el)))
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      d1[k] = pack_vec<T>(f_dt + k * V);
      d2[k] = pack_vec<T>(f_dg + k * V);
    }
    carry = row_start ? cb : fmaf(ca, carry, cb);
  }
}

// Segments per row for the split path (1 = not used).  Segments are fixed
// at kSegChunks chunks (32 KiB per tensor).  Measured on B200 (fp32 and
// bf16, L = 16K..64K): splitting wins only when rows are few and long --
// 8 rows: +66%, 64 rows x 64K fp32: +6% -- and loses once the tiles exceed
// about two waves or a row has fewer than 4 segments, so it is used only
// when rows * segments <= 2 * slots and segments >= 4.
int split_segments(int64_t rows, int64_t seqlen, int dtype, int slots) {
  const int es = dtype_size(dtype);
  const int64_t seg = (int64_t)kSegChunks * kThreads * kSplitNV * (16 / es);
  if (rows <= 0 || seqlen < 4 * seg) return 1;
  const int64_t p = seqlen / seg;
  if (rows * p > 2 * (int64_t)slots) return 1;
  return (int)p;
}

int split_slots(int dtype, int num_sms) {
  static int occ_cache[3][64] = {{0}};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return num_sms * 4;
  int& occ = occ_cache[dtype][dev];
  if (occ == 0) {
    int n = 0;
    cudaError_t e = cudaSuccess;
    switch (dtype) {
      case kF32:
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, scan_split_kernel<float, false>, kThreads, kSplitSmem);
        break;
      case kF16:
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, scan_split_kernel<__half, false>, kThreads, kSplitSmem);
        break;
      default:
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, scan_split_kernel<__nv_bfloat16, false>, kThreads, kSplitSmem);
    }
    // Before the dynamic-smem opt-in the query can report 0; the ring fits 3.
    occ = (e == cudaSuccess && n > 0) ? n : 3;
  }
  return num_sms * occ;
}

int64_t split_workspace_bytes(int64_t rows, int p) {
  return p > 1 ? 256 + (int64_t)sizeof(SegStatus) * rows * p : 0;
}

// Segments per row for the split-row fused backward (1 = not used): same
// rule as the forward (rows * segments within two waves, at least 4
// segments per row), with segments of kSegChunks one-vector chunks.
// FPSCAN_B200_SPLIT_BWD_WAVES raises the wave limit for measurement: at 512
// rows of 65536 (8 segments per row, ~7 waves) the split kernel ran 3.6 TB/s
// (bf16) / 3.7 TB/s (fp32) against 5.2 / 5.3 for one CTA per row, since each
// tile stages, scans, looks back and stores in turn with no overlap.
int split_bwd_segments(int64_t rows, int64_t seqlen, int dtype, int num_sms) {
  const int es = dtype_size(dtype);
  const int64_t seg = (int64_t)kSegChunks * kThreads * kSplitBwdNV * (16 / es);
  if (rows <= 0 || seqlen < 4 * seg) return 1;
  const int64_t p = seqlen / seg;
  int occ = 4;
  {
    static int occ_cache[3][64] = {{0}};
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < 64) {
      int& oc = occ_cache[dtype][dev];
      if (oc == 0) {
        int n = 0;
        cudaError_t e;
        switch (dtype) {
          case kF32:
            cudaFuncSetAttribute(scan_split_bwd_kernel<float>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, kSplitBwdSmem);
            e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, scan_split_bwd_kernel<float>,
                                                              kThreads, kSplitBwdSmem);
            break;
          case kF16:
            cudaFuncSetAttribute(scan_split_bwd_kernel<__half>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, kSplitBwdSmem);
            e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, scan_split_bwd_kernel<__half>,
                                                              kThreads, kSplitBwdSmem);
            break;
          default:
            cudaFuncSetAttribute(scan_split_bwd_kernel<__nv_bfloat16>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, kSplitBwdSmem);
            e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                &n, scan_split_bwd_kernel<__nv_bfloat16>, kThreads, kSplitBwdSmem);
        }
        if (e != cudaSuccess) cudaGetLastError();
        oc = (e == cudaSuccess && n > 0) ? n : 4;
      }
      occ = oc;
    }
  }
  static const int waves = [] {
    const char* v = getenv("FPSCAN_B200_SPLIT_BWD_WAVES");
    const int w = v ? atoi(v) : 2;
    return w > 0 ? w : 2;
  }();
  if (rows * p > (int64_t)waves * num_sms * occ) return 1;
  return (int)p;
}

static uint32_t next_epoch() {
  static std::atomic<uint32_t> ctr{0};
  uint32_t e;
  do {
    e = (ctr.fetch_add(1, std::memory_order_relaxed) + 1) & 0x7fffffffu;
  } while (e == 0);
  return e;
}

template <typename T, bool REV>
static cudaError_t launch_split_t(const SplitArgs& a) {
  auto kern = scan_split_kernel<T, REV>;
  static int configured[64] = {0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSplitSmem);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) configured[dev] = 1;
  }
  e = cudaMemsetAsync(a.workspace, 0, sizeof(unsigned long long), a.stream);
  if (e != cudaSuccess) return e;
  SplitKParams p;
  p.gates = a.gates;
  p.tokens = a.tokens;
  p.out = a.out;
  p.counter = static_cast<unsigned long long*>(a.workspace);
  p.status = reinterpret_cast<SegStatus*>(static_cast<char*>(a.workspace) + 256);
  p.rows = a.rows;
  p.lg = ilog2_host(a.seqlen);
  p.lgp = ilog2_host(a.segments);
  p.epoch = next_epoch();
  const int64_t tiles = a.rows * a.segments;
  return launch_pdl(kern, (unsigned)tiles, kThreads, kSplitSmem, a.stream, p);
}

template <typename T>
static cudaError_t launch_split_bwd_t(const SplitBwdArgs& a) {
  auto kern = scan_split_bwd_kernel<T>;
  static int configured[64] = {0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSplitBwdSmem);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) configured[dev] = 1;
  }
  e = cudaMemsetAsync(a.workspace, 0, sizeof(unsigned long long), a.stream);
  if (e != cudaSuccess) return e;
  SplitBwdKParams p;
  p.gates = a.gates;
  p.y = a.y;
  p.gout = a.grad_out;
  p.dgates = a.dgates;
  p.dtok = a.dtokens;
  p.counter = static_cast<unsigned long long*>(a.workspace);
  p.status = reinterpret_cast<SegStatus*>(static_cast<char*>(a.workspace) + 256);
  p.rows = a.rows;
  p.lg = ilog2_host(a.seqlen);
  p.lgp = ilog2_host(a.segments);
  p.epoch = next_epoch();
  const int64_t tiles = a.rows * a.segments;
  return launch_pdl(kern, (unsigned)tiles, kThreads, kSplitBwdSmem, a.stream, p);
}

cudaError_t launch_split_bwd(const SplitBwdArgs& a) {
  switch (a.dtype) {
    case kF32:
      return launch_split_bwd_t<float>(a);
    case kF16:
      return launch_split_bwd_t<__half>(a);
    case kBF16:
      return launch_split_bwd_t<__nv_bfloat16>(a);
    default:
      return cudaErrorInvalidValue;
  }
}

cudaError_t launch_split(const SplitArgs& a) {
  switch (a.dtype) {
    case kF32:
      return a.reverse ? launch_split_t<float, true>(a) : launch_split_t<float, false>(a);
    case kF16:
      return a.reverse ? launch_split_t<__half, true>(a) : launch_split_t<__half, false>(a);
    case kBF16:
      return a.reverse ? launch_split_t<__nv_bfloat16, true>(a)
                       : launch_split_t<__nv_bfloat16, false>(a);
    default:
      return cudaErrorInvalidValue;
  }
}

}  // namespace fpscan
