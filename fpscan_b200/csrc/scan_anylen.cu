// Forward / reverse scan and fused backward for ANY seqlen >= 1 (not only the
// reference's powers of two in [32, 65536], csrc/full_scan/full_scan.cu:207-233),
// sm_100a.
//
// The (rows, L) tensor is treated as one flat stream of rows*L elements in
// which every row start is a segment head.  Each CTA owns a contiguous run of
// whole rows (one wave of tiles, as in scan_fwd.cu) and streams it in chunks
// aligned to 16-byte vectors of the flat buffer, so row boundaries fall
// anywhere inside a thread's elements.  The scan is a segmented scan of the
// affine maps (A, B): a head discards everything before it (zero initial
// state; the head's gate is ignored like the reference's forced 1.0 at
// full_scan.cu:96).  Discarding is a select, never a multiplication by 0, so
// an inf/NaN state of one row cannot leak into the next.
//   * thread: serial segmented scan of its E elements (head bitmask from the
//     element positions, tracked incrementally: one 64-bit modulo per thread
//     per launch);
//   * warp: Hillis-Steele scan of the thread totals where lane i only takes
//     lanes at or after the last head lane <= i (from a ballot of the lanes
//     that hold a head);
//   * block: the same over the 8 warp totals, done redundantly by each warp;
//   * chunk carry: fp32 state carried across chunks.
// Elements of neighbouring tiles that share a 16-byte vector with this tile
// are read (their rows end with a head before ours) but never written:
// partial vectors are stored element by element.  The last partial vector of
// the buffer (rows*L not a multiple of the vector width) is not staged by
// the bulk copies; the one thread that owns it reads it from global memory.
#include <cstdlib>

#include "common.cuh"
#include "internal.h"

namespace fpscan {

namespace {

template <typename T, int NV>
struct AnyCfg {
  static constexpr int kStages = NV == 1 ? 4 : 3;
  static constexpr int kMinBlocks = 3;
  // the backward with two vectors per thread gets a 2-CTA register budget
  // (it spills under the 3-CTA one)
  static constexpr int kBwdMinBlocks = NV == 2 ? 2 : 3;
  static constexpr int SV = kThreads * NV;  // 16-byte vectors per chunk
  static constexpr int fwd_smem() { return kStages * 2 * SV * 16; }
  static constexpr int kBwdStages = NV == 1 ? 4 : 3;
  static constexpr int bwd_smem() { return kBwdStages * 16 * (3 * SV + 2); }
};

struct AnyKParams {
  const void* gates;
  const void* tokens;   // forward: tokens; backward: grad_out
  const void* y;        // backward: forward output
  void* out;            // forward: y; backward: dtokens
  void* out2;           // backward: dgates
  int64_t rows;
  int64_t rows_per_tile;
  int64_t L;
  int64_t n_total;      // rows * L
  int64_t ch_mod_L;     // chunk length mod L
};

// Segmented inclusive scan of (a, b) across the warp: lane i combines only
// with lanes >= the last lane <= i whose value holds a head (`heads` = ballot
// of those lanes).  Returns whether a head is among lanes 0..i.
__device__ __forceinline__ bool warp_seg_scan(float& a, float& b, int lane, unsigned heads) {
  const unsigned upto = heads & (0xffffffffu >> (31 - lane));
  const int ss = upto ? 31 - __clz(upto) : -1;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const float pa = __shfl_up_sync(0xffffffffu, a, d);
    const float pb = __shfl_up_sync(0xffffffffu, b, d);
    if (lane - d >= ss && lane >= d) {
      b = fmaf(pb, a, b);
      a = pa * a;
    }
  }
  return upto != 0;
}

// Compose an earlier map (f0, a0, b0) with a later one (f1, a1, b1).
__device__ __forceinline__ void seg_compose(bool f0, float a0, float b0, bool& f1, float& a1,
                                            float& b1) {
  if (!f1) {
    b1 = fmaf(b0, a1, b1);
    a1 = a0 * a1;
    f1 = f0;
  }
}

// Thread's exclusive prefix within the chunk from its in-warp exclusive
// prefix (ef, ea, eb) and the warp totals in `wt` (x = A, y = B, z = head
// flag); also returns the chunk total (cf, ca, cb).  Every warp scans the
// kWarps totals in its lanes 0..kWarps-1.
__device__ __forceinline__ void block_seg_prefix(const float4* wt, int lane, int warp, bool& ef,
                                                 float& ea, float& eb, bool& cf, float& ca,
                                                 float& cb) {
  const float4 t = wt[lane & (kWarps - 1)];
  float a = t.x, b = t.y;
  const unsigned heads = __ballot_sync(0xffffffffu, t.z != 0.f) & ((1u << kWarps) - 1);
  const int sl = lane & (kWarps - 1);
  const unsigned upto = heads & ((2u << sl) - 1);
  const int ss = upto ? 31 - __clz(upto) : -1;
#pragma unroll
  for (int d = 1; d < kWarps; d <<= 1) {
    const float pa = __shfl_up_sync(0xffffffffu, a, d);
    const float pb = __shfl_up_sync(0xffffffffu, b, d);
    if (sl - d >= ss && sl >= d) {
      b = fmaf(pb, a, b);
      a = pa * a;
    }
  }
  const int src = (warp - 1) & (kWarps - 1);
  const float wa = __shfl_sync(0xffffffffu, a, src);
  const float wb = __shfl_sync(0xffffffffu, b, src);
  ca = __shfl_sync(0xffffffffu, a, kWarps - 1);
  cb = __shfl_sync(0xffffffffu, b, kWarps - 1);
  cf = heads != 0;
  if (warp != 0) {
    const bool wf = (heads & ((1u << warp) - 1)) != 0;
    seg_compose(wf, wa, wb, ef, ea, eb);
  }
}

// Stores E fp32 values (memory order) of the thread's NV vectors starting at
// element e0, only for elements inside [ts, te).
template <typename T, int NV>
__device__ __forceinline__ void store_masked(T* dst, int64_t e0, int64_t ts, int64_t te,
                                             const float* f FPSCAN_DEBUG_ONLY(, int64_t n)) {
  constexpr int V = Elem<T>::kVec;
#pragma unroll
  for (int q = 0; q < NV; ++q) {
    const int64_t vs = e0 + q * V;
    if (vs >= ts && vs + V <= te) {
      FPSCAN_DEBUG_ONLY(if (in_bounds(dst + vs, 16, dst, dst + n)))
      reinterpret_cast<uint4*>(dst + vs)[0] = pack_vec<T>(f + q * V);
    } else {
#pragma unroll
      for (int j = 0; j < V; ++j) {
        const int64_t t = vs + j;
        if (t >= ts && t < te FPSCAN_DEBUG_ONLY(
                                  && in_bounds<sizeof(T)>(dst + t, sizeof(T), dst, dst + n)))
          dst[t] = Elem<T>::store(f[q * V + j]);
      }
    }
  }
}

// Head bitmasks of a thread's E elements (memory order) from the position
// within its row of the first element: bit j of `first` / `last` is set when
// element j starts / ends a row.  For L >= E a thread holds at most one row
// start after its first element and at most one row end, so the masks cost a
// few scalar operations; shorter rows take the per-element loop.
template <int E>
__device__ __forceinline__ void row_masks(int64_t pos0, int64_t L, unsigned& first,
                                          unsigned& last) {
  if (L >= E) {
    const int64_t to_end = L - 1 - pos0;  // elements after the first one in its row
    first = (pos0 == 0 ? 1u : 0u) | (to_end < E - 1 ? 2u << to_end : 0u);
    last = to_end < E ? 1u << to_end : 0u;
    return;
  }
  first = last = 0;
  int64_t p = pos0;
#pragma unroll
  for (int j = 0; j < E; ++j) {
    if (p == 0) first |= 1u << j;
    if (p == L - 1) last |= 1u << j;
    p = (p + 1 == L) ? 0 : p + 1;
  }
}

// ------------------------------------------------------------------ forward
template <typename T, int NV, bool REV>
__global__ void __launch_bounds__(kThreads, (AnyCfg<T, NV>::kMinBlocks))
    scan_anylen_fwd_kernel(const AnyKParams p) {
  constexpr int V = Elem<T>::kVec;
  constexpr int E = V * NV;
  constexpr int CH = kThreads * E;
  constexpr int S = AnyCfg<T, NV>::kStages;
  constexpr int SV = AnyCfg<T, NV>::SV;

  extern __shared__ __align__(128) uint4 dsm[];
  uint4 (*s_g)[SV] = reinterpret_cast<uint4 (*)[SV]>(dsm);
  uint4 (*s_x)[SV] = reinterpret_cast<uint4 (*)[SV]>(dsm + S * SV);
  __shared__ __align__(8) uint64_t s_bar[S];
  __shared__ float4 s_wt[2][kWarps];

  const T* __restrict__ gates = static_cast<const T*>(p.gates);
  const T* __restrict__ tokens = static_cast<const T*>(p.tokens);
  T* out = static_cast<T*>(p.out);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t L = p.L, N = p.n_total;
  const int64_t row0 = (int64_t)blockIdx.x * p.rows_per_tile;
  const int64_t nrows = min(p.rows_per_tile, p.rows - row0);
  if (nrows <= 0) return;
  const int64_t ts = row0 * L, te = (row0 + nrows) * L;  // tile elements
  const int64_t as = ts - ts % V;                          // aligned chunk origin
  const int64_t te_up = (te + V - 1) / V * V;
  const int64_t n_floor = N / V * V;                       // end of whole vectors
  const int64_t nck = (te - as + CH - 1) / CH;

  if (tid == 0) {
#pragma unroll
    for (int s = 0; s < S; ++s) mbar_init(&s_bar[s], 1);
    fence_mbar_init();
  }
  __syncthreads();
  pdl_wait();  // the previous kernel in the stream is complete from here on
  pdl_launch_dependents();

  int64_t issued = 0;
  auto issue = [&](int64_t k) {
    const int64_t mc = REV ? nck - 1 - k : k;
    const int64_t cs = as + mc * CH;
    const int64_t ce = min(min(cs + CH, te_up), n_floor);
    const uint32_t bytes = ce > cs ? (uint32_t)((ce - cs) * (int64_t)sizeof(T)) : 0u;
    const int s = (int)(k % S);
    // debug builds: a copy outside its tensor is skipped, the stage completes
    FPSCAN_DEBUG_ONLY(
        if (bytes && (!in_bounds(gates + cs, bytes, gates, gates + N) ||
                      !in_bounds(tokens + cs, bytes, tokens, tokens + N))) {
          mbar_expect_tx(&s_bar[s], 0u);
          return;
        })
    mbar_expect_tx(&s_bar[s], 2u * bytes);
    if (bytes) {
      bulk_g2s(s_g[s], gates + cs, bytes, &s_bar[s]);
      bulk_g2s(s_x[s], tokens + cs, bytes, &s_bar[s]);
    }
  };
  if (tid == 0) {
    for (; issued < min((int64_t)S, nck); ++issued) issue(issued);
  }

  const int vi = REV ? kThreads - 1 - tid : tid;
  // Position within its row of the thread's first element in the first
  // processed chunk; advanced by one chunk (mod L) per step.
  int64_t pos;
  {
    const int64_t mc0 = REV ? nck - 1 : 0;
    pos = (as + mc0 * CH + (int64_t)vi * E) % L;
  }
  float carry = 0.f;
  int64_t k = 0;
  int s = 0;
  uint32_t phase = 0;
  bool aborted = false;

  for (; k < nck; ++k) {
    const int64_t mc = REV ? nck - 1 - k : k;
    const int64_t cs = as + mc * CH;
    const int64_t e0 = cs + (int64_t)vi * E;
    const bool valid = e0 < te && e0 + E > ts;
    const bool slow = valid && e0 + E > n_floor;  // owns the buffer's partial last vector

    const bool ok = mbar_wait_bounded(&s_bar[s], phase);

    unsigned first_m, last_m;
    row_masks<E>(pos, L, first_m, last_m);
    const unsigned head_m = REV ? last_m : first_m;

    float a[E], b[E];
    unsigned incl = 0;  // bit i: a head among processing-order elements 0..i
    if (valid) {
      Vec16<T> gv[NV], xv[NV];
      if (!slow) {
        uint4 rg[NV], rx[NV];
        lds_vecs<NV>(&s_g[s][vi * NV], rg);
        lds_vecs<NV>(&s_x[s][vi * NV], rx);
#pragma unroll
        for (int q = 0; q < NV; ++q) {
          gv[q].raw = rg[q];
          xv[q].raw = rx[q];
        }
      } else {
#pragma unroll
        for (int j = 0; j < E; ++j) {
          const int64_t t = e0 + j;
          gv[j / V].e[j % V] = t < N ? gates[t] : Elem<T>::store(1.f);
          xv[j / V].e[j % V] = t < N ? tokens[t] : Elem<T>::store(0.f);
        }
      }
      if (head_m == 0) {  // no row boundary inside the thread's elements
#pragma unroll
        for (int i = 0; i < E; ++i) {
          const int j = REV ? E - 1 - i : i;
          const float g = Elem<T>::load(gv[j / V].e[j % V]);
          const float x = Elem<T>::load(xv[j / V].e[j % V]);
          a[i] = i == 0 ? g : a[i - 1] * g;
          b[i] = i == 0 ? x : fmaf(b[i - 1], g, x);
        }
      } else {
      bool f = false;
#pragma unroll
      for (int i = 0; i < E; ++i) {
        const int j = REV ? E - 1 - i : i;
        const float g = Elem<T>::load(gv[j / V].e[j % V]);
        const float x = Elem<T>::load(xv[j / V].e[j % V]);
        if ((head_m >> j) & 1u) {
          a[i] = 1.f;
          b[i] = x;
          f = true;
        } else if (i == 0) {
          a[0] = g;
          b[0] = x;
        } else {
          a[i] = a[i - 1] * g;
          b[i] = fmaf(b[i - 1], g, x);
        }
        if (f) incl |= 1u << i;
      }
      }
    } else {
#pragma unroll
      for (int i = 0; i < E; ++i) {
        a[i] = 1.f;
        b[i] = 0.f;
      }
    }

    // warp level
    const bool tf = incl != 0;
    const unsigned heads = __ballot_sync(0xffffffffu, tf);
    float ta = a[E - 1], tb = b[E - 1];
    const bool tf_incl = warp_seg_scan(ta, tb, lane, heads);
    float ea = __shfl_up_sync(0xffffffffu, ta, 1);
    float eb = __shfl_up_sync(0xffffffffu, tb, 1);
    bool ef = (heads & ((1u << lane) - 1)) != 0;
    if (lane == 0) {
      ea = 1.f;
      eb = 0.f;
    }
    const int buf = (int)(k & 1);
    if (lane == 31) s_wt[buf][warp] = make_float4(ta, tb, tf_incl ? 1.f : 0.f, 0.f);

    if (__syncthreads_or(!ok)) {
      aborted = true;
      break;
    }
    if (tid == 0 && issued < nck) {
      issue(issued);
      ++issued;
    }

    bool cf;
    float ca, cb;
    block_seg_prefix(s_wt[buf], lane, warp, ef, ea, eb, cf, ca, cb);
    // y just before the thread's first element (processing order); only
    // used by elements not preceded by a head inside the thread
    const float state = ef ? eb : fmaf(ea, carry, eb);

    if (valid) {
      float f[E];  // memory order
      if (incl == 0) {
#pragma unroll
        for (int i = 0; i < E; ++i) f[REV ? E - 1 - i : i] = fmaf(a[i], state, b[i]);
      } else {
#pragma unroll
        for (int i = 0; i < E; ++i)
          f[REV ? E - 1 - i : i] = ((incl >> i) & 1u) ? b[i] : fmaf(a[i], state, b[i]);
      }
      store_masked<T, NV>(out, e0, ts, te, f FPSCAN_DEBUG_ONLY(, N));
    }

    carry = cf ? cb : fmaf(ca, carry, cb);
    if (REV) {
      pos -= p.ch_mod_L;
      if (pos < 0) pos += L;
    } else {
      pos += p.ch_mod_L;
      if (pos >= L) pos -= L;
    }
    if (++s == S) {
      s = 0;
      phase ^= 1u;
    }
  }

  if (aborted && tid == 0) {
    for (int64_t kk = k; kk < issued; ++kk)
      mbar_wait_bounded(&s_bar[kk % S], (uint32_t)((kk / S) & 1));
  }
}

// ------------------------------------------------------------------ backward
// dtokens[t] = grad_out[t] + gates[t+1] * dtokens[t+1]   (t not a row's last)
// dgates[t]  = dtokens[t] * y[t-1]                         (0 at a row's first)
// One reverse pass reading gates, y, grad_out once; gates[t+1] and y[t-1]
// at a thread's edges come from one extra staged vector after the gates chunk
// and before the y chunk.
template <typename T, int NV>
__global__ void __launch_bounds__(kThreads, (AnyCfg<T, NV>::kBwdMinBlocks))
    scan_anylen_bwd_kernel(const AnyKParams p) {
  constexpr int V = Elem<T>::kVec;
  constexpr int E = V * NV;
  constexpr int CH = kThreads * E;
  constexpr int S = AnyCfg<T, NV>::kBwdStages;
  constexpr int SV = AnyCfg<T, NV>::SV;
  constexpr int GS = SV + 1, YS = SV + 1;

  extern __shared__ __align__(128) uint4 dsm[];
  uint4* s_g = dsm;             // [S][GS]
  uint4* s_go = s_g + S * GS;   // [S][SV]
  uint4* s_y = s_go + S * SV;   // [S][YS]
  __shared__ __align__(8) uint64_t s_bar[S];
  __shared__ float4 s_wt[2][kWarps];

  const T* __restrict__ gates = static_cast<const T*>(p.gates);
  const T* __restrict__ gout = static_cast<const T*>(p.tokens);
  const T* __restrict__ y = static_cast<const T*>(p.y);
  T* dtok = static_cast<T*>(p.out);
  T* dgates = static_cast<T*>(p.out2);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t L = p.L, N = p.n_total;
  const int64_t row0 = (int64_t)blockIdx.x * p.rows_per_tile;
  const int64_t nrows = min(p.rows_per_tile, p.rows - row0);
  if (nrows <= 0) return;
  const int64_t ts = row0 * L, te = (row0 + nrows) * L;
  const int64_t as = ts - ts % V;
  const int64_t te_up = (te + V - 1) / V * V;
  const int64_t n_floor = N / V * V;
  const int64_t nck = (te - as + CH - 1) / CH;

  if (tid == 0) {
#pragma unroll
    for (int s = 0; s < S; ++s) mbar_init(&s_bar[s], 1);
    fence_mbar_init();
  }
  __syncthreads();
  pdl_wait();  // the previous kernel in the stream is complete from here on
  pdl_launch_dependents();

  int64_t issued = 0;
  auto issue = [&](int64_t k) {
    const int64_t mc = nck - 1 - k;
    const int64_t cs = as + mc * CH;
    const int64_t ce = min(min(cs + CH, te_up), n_floor);
    const int s = (int)(k % S);
    if (ce <= cs) {  // only the buffer's partial last vector: read from global
      mbar_expect_tx(&s_bar[s], 0u);
      return;
    }
    const uint32_t bytes = (uint32_t)((ce - cs) * (int64_t)sizeof(T));
    const int64_t ge = min(min(cs + CH + V, te_up), n_floor);
    const uint32_t g_bytes = (uint32_t)((ge - cs) * (int64_t)sizeof(T));
    const bool y_halo = cs > as;
    const uint32_t y_bytes = bytes + (y_halo ? 16u : 0u);
    // debug builds: a copy outside its tensor is skipped, the stage completes
    FPSCAN_DEBUG_ONLY(
        if (!in_bounds(gates + cs, g_bytes, gates, gates + N) ||
            !in_bounds(gout + cs, bytes, gout, gout + N) ||
            !in_bounds(y_halo ? y + cs - V : y + cs, y_bytes, y, y + N)) {
          mbar_expect_tx(&s_bar[s], 0u);
          return;
        })
    mbar_expect_tx(&s_bar[s], g_bytes + bytes + y_bytes);
    bulk_g2s(s_g + s * GS, gates + cs, g_bytes, &s_bar[s]);
    bulk_g2s(s_go + s * SV, gout + cs, bytes, &s_bar[s]);
    if (y_halo)
      bulk_g2s(s_y + s * YS, y + cs - V, y_bytes, &s_bar[s]);
    else
      bulk_g2s(s_y + s * YS + 1, y + cs, y_bytes, &s_bar[s]);
  };
  if (tid == 0) {
    for (; issued < min((int64_t)S, nck); ++issued) issue(issued);
  }

  const int vi = kThreads - 1 - tid;
  int64_t pos = (as + (nck - 1) * CH + (int64_t)vi * E) % L;
  float carry = 0.f;
  int64_t k = 0;
  int s = 0;
  uint32_t phase = 0;
  bool aborted = false;

  for (; k < nck; ++k) {
    const int64_t mc = nck - 1 - k;
    const int64_t cs = as + mc * CH;
    const int64_t e0 = cs + (int64_t)vi * E;
    const bool valid = e0 < te && e0 + E > ts;
    // Threads whose data or right halo reach the buffer's partial last
    // vector read from global memory.
    const bool slow = valid && e0 + E + V > n_floor;

    const bool ok = mbar_wait_bounded(&s_bar[s], phase);

    unsigned first_m, last_m;
    row_masks<E>(pos, L, first_m, last_m);

    Vec16<T> gv[NV], gov[NV], yv[NV];
    float g_next = 1.f, y_before = 0.f;
    if (valid) {
      if (!slow) {
        uint4 rg[NV], rgo[NV], ry[NV];
        const uint4* sg = s_g + s * GS + vi * NV;
        const uint4* sy = s_y + s * YS + 1 + vi * NV;
        lds_vecs<NV>(sg, rg);
        lds_vecs<NV>(s_go + s * SV + vi * NV, rgo);
        lds_vecs<NV>(sy, ry);
#pragma unroll
        for (int q = 0; q < NV; ++q) {
          gv[q].raw = rg[q];
          gov[q].raw = rgo[q];
          yv[q].raw = ry[q];
        }
        if (!((last_m >> (E - 1)) & 1u))
          g_next = Elem<T>::load(reinterpret_cast<const T*>(sg + NV)[0]);
        if (!(first_m & 1u)) y_before = Elem<T>::load(reinterpret_cast<const T*>(sy)[-1]);
      } else {
#pragma unroll
        for (int j = 0; j < E; ++j) {
          const int64_t t = e0 + j;
          gv[j / V].e[j % V] = t < N ? gates[t] : Elem<T>::store(1.f);
          gov[j / V].e[j % V] = t < N ? gout[t] : Elem<T>::store(0.f);
          yv[j / V].e[j % V] = t < N ? y[t] : Elem<T>::store(0.f);
        }
        if (!((last_m >> (E - 1)) & 1u) && e0 + E < N) g_next = Elem<T>::load(gates[e0 + E]);
        if (!(first_m & 1u) && e0 > 0) y_before = Elem<T>::load(y[e0 - 1]);
      }
    }

    float a[E], b[E];
    unsigned incl = 0;
    if (valid && last_m == 0) {  // no row end inside the thread's elements
#pragma unroll
      for (int i = 0; i < E; ++i) {
        const int j = E - 1 - i;
        const float g = (j == E - 1) ? g_next : Elem<T>::load(gv[(j + 1) / V].e[(j + 1) % V]);
        const float x = Elem<T>::load(gov[j / V].e[j % V]);
        a[i] = i == 0 ? g : a[i - 1] * g;
        b[i] = i == 0 ? x : fmaf(b[i - 1], g, x);
      }
    } else if (valid) {
      bool f = false;
#pragma unroll
      for (int i = 0; i < E; ++i) {
        const int j = E - 1 - i;
        const float g = (j == E - 1) ? g_next : Elem<T>::load(gv[(j + 1) / V].e[(j + 1) % V]);
        const float x = Elem<T>::load(gov[j / V].e[j % V]);
        if ((last_m >> j) & 1u) {
          a[i] = 1.f;
          b[i] = x;
          f = true;
        } else if (i == 0) {
          a[0] = g;
          b[0] = x;
        } else {
          a[i] = a[i - 1] * g;
          b[i] = fmaf(b[i - 1], g, x);
        }
        if (f) incl |= 1u << i;
      }
    } else {
#pragma unroll
      for (int i = 0; i < E; ++i) {
        a[i] = 1.f;
        b[i] = 0.f;
      }
    }

    const unsigned heads = __ballot_sync(0xffffffffu, incl != 0);
    float ta = a[E - 1], tb = b[E - 1];
    const bool tf_incl = warp_seg_scan(ta, tb, lane, heads);
    float ea = __shfl_up_sync(0xffffffffu, ta, 1);
    float eb = __shfl_up_sync(0xffffffffu, tb, 1);
    bool ef = (heads & ((1u << lane) - 1)) != 0;
    if (lane == 0) {
      ea = 1.f;
      eb = 0.f;
    }
    const int buf = (int)(k & 1);
    if (lane == 31) s_wt[buf][warp] = make_float4(ta, tb, tf_incl ? 1.f : 0.f, 0.f);

    if (__syncthreads_or(!ok)) {
      aborted = true;
      break;
    }
    if (tid == 0 && issued < nck) {
      issue(issued);
      ++issued;
    }

    bool cf;
    float ca, cb;
    block_seg_prefix(s_wt[buf], lane, warp, ef, ea, eb, cf, ca, cb);
    const float state = ef ? eb : fmaf(ea, carry, eb);

    if (valid) {
      float f_dt[E], f_dg[E];  // memory order
      if ((incl | first_m) == 0) {
#pragma unroll
        for (int i = 0; i < E; ++i) {
          const int j = E - 1 - i;
          const float dt = fmaf(a[i], state, b[i]);
          const float yp = j == 0 ? y_before : Elem<T>::load(yv[(j - 1) / V].e[(j - 1) % V]);
          f_dt[j] = dt;
          f_dg[j] = dt * yp;
        }
      } else {
#pragma unroll
        for (int i = 0; i < E; ++i) {
          const int j = E - 1 - i;
          const float dt = ((incl >> i) & 1u) ? b[i] : fmaf(a[i], state, b[i]);
          const float yp =
              ((first_m >> j) & 1u)
                  ? 0.f
                  : (j == 0 ? y_before : Elem<T>::load(yv[(j - 1) / V].e[(j - 1) % V]));
          f_dt[j] = dt;
          f_dg[j] = dt * yp;
        }
      }
      store_masked<T, NV>(dtok, e0, ts, te, f_dt FPSCAN_DEBUG_ONLY(, N));
      store_masked<T, NV>(dgates, e0, ts, te, f_dg FPSCAN_DEBUG_ONLY(, N));
    }

    carry = cf ? cb : fmaf(ca, carry, cb);
    pos -= p.ch_mod_L;
    if (pos < 0) pos += L;
    if (++s == S) {
      s = 0;
      phase ^= 1u;
    }
  }

  if (aborted && tid == 0) {
    for (int64_t kk = k; kk < issued; ++kk)
      mbar_wait_bounded(&s_bar[kk % S], (uint32_t)((kk / S) & 1));
  }
}

template <typename Kern>
static cudaError_t launch_one_wave(Kern kern, int smem, const AnyArgs& a, AnyKParams p,
                                   int* occ_cache) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  int occ = (dev >= 0 && dev < 64) ? occ_cache[dev] : 0;
  if (occ == 0) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kThreads, smem) != cudaSuccess ||
        occ < 1)
      occ = 1;
    if (dev >= 0 && dev < 64) occ_cache[dev] = occ;
  }
  // Tiles: 8 waves' worth of static row tiles, handed out by the block
  // scheduler as CTAs finish -- the balancing that claimed row units give
  // the power-of-two kernels, without per-chunk unit bounds in shared
  // memory (which cost more than they saved here).  Measured (GB/s, fwd /
  // rev / bwd, one wave -> 8 waves): fp32 (8, 2048, 8191) 5394 / 5584 /
  // 5492 -> 6563 / 6587 / 5548; bf16 (16, 5120, 16383) 5727 / 5541 / 5434
  // -> 5858 / 5674 / 5662; fp32 (2, 256, 100000) reverse 4299 -> 4827;
  // bf16 (8, 2048, 8191) forward 5410 -> 5214 (the one loss).
  // FPSCAN_B200_ANY_WAVES overrides the number of waves.
  static const int64_t waves = [] {
    const char* v = getenv("FPSCAN_B200_ANY_WAVES");
    return v ? (int64_t)atoi(v) : (int64_t)8;
  }();
  const int64_t slots = (int64_t)a.num_sms * occ * (waves > 0 ? waves : 1);
  int64_t rpt = (a.rows + slots - 1) / slots;
  if (rpt < 1) rpt = 1;
  const int64_t tiles = (a.rows + rpt - 1) / rpt;
  p.rows = a.rows;
  p.rows_per_tile = rpt;
  p.L = a.seqlen;
  p.n_total = a.rows * a.seqlen;
  return launch_pdl(kern, (unsigned)tiles, kThreads, smem, a.stream, p);
}

template <typename T, int NV>
static cudaError_t launch_any_t(const AnyArgs& a) {
  constexpr int CH = kThreads * Elem<T>::kVec * NV;
  AnyKParams p{};
  p.gates = a.gates;
  p.ch_mod_L = CH % a.seqlen;
  if (a.backward) {
    static int occ_b[64] = {0};
    p.tokens = a.grad_out;
    p.y = a.y;
    p.out = a.dtokens;
    p.out2 = a.dgates;
    return launch_one_wave(scan_anylen_bwd_kernel<T, NV>, AnyCfg<T, NV>::bwd_smem(), a, p, occ_b);
  }
  p.tokens = a.tokens;
  p.out = a.out;
  if (a.reverse) {
    static int occ_r[64] = {0};
    return launch_one_wave(scan_anylen_fwd_kernel<T, NV, true>, AnyCfg<T, NV>::fwd_smem(), a, p,
                           occ_r);
  }
  static int occ_f[64] = {0};
  return launch_one_wave(scan_anylen_fwd_kernel<T, NV, false>, AnyCfg<T, NV>::fwd_smem(), a, p,
                         occ_f);
}

template <typename T>
static cudaError_t launch_any_nv(const AnyArgs& a) {
  return a.nv == 2 ? launch_any_t<T, 2>(a) : launch_any_t<T, 1>(a);
}

}  // namespace

cudaError_t launch_anylen(const AnyArgs& a) {
  switch (a.dtype) {
    case kF32:
      return launch_any_nv<float>(a);
    case kF16:
      return launch_any_nv<__half>(a);
    case kBF16:
      return launch_any_nv<__nv_bfloat16>(a);
    default:
      return cudaErrorInvalidValue;
  }
}

}  // namespace fpscan
