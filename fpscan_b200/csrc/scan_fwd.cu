// Forward / reverse linear-recurrence scan over the last axis of a
// (rows, L) row-major tensor, sm_100a.
//
// Replaces the reference kernel scan<> (csrc/full_scan/full_scan.cu:50-177)
// with a different design:
//   * the grid is one wave (SMs x resident CTAs); each CTA streams units of
//     whole consecutive rows -- its first unit by index, the rest claimed from
//     a per-launch counter (sched.cuh), or one static tile -- chunk by chunk
//     through a kStages-deep shared-memory ring filled by non-multicast
//     cp.async.bulk copies completing on mbarriers, so its pipeline runs
//     across row and unit boundaries without draining;
//   * each thread owns NV consecutive 16-byte vectors of a chunk (4*NV fp32 or
//     8*NV half values): in-register serial scan, warp-shuffle Hillis-Steele
//     scan of the thread totals, then a lane-parallel scan of the
//     (double-buffered) warp totals done redundantly by every warp -- one
//     __syncthreads per chunk;
//   * rows shorter than a chunk are packed several to a chunk and scanned as
//     independent segments (row boundaries coincide with power-of-two thread
//     groups); rows longer than a chunk carry their fp32 state across chunks;
//   * 64-bit offsets, shifts and masks only (seqlen is a power of two); any
//     number of rows.
// Optional per-row initial state (`init`) and per-row carry-out
// (A = product of all gates of the row, B = final state) serve the
// sequence-sharded multi-GPU mode.  Without `init` the gate of a row's first
// element is ignored, exactly like the reference's forced 1.0
// (csrc/full_scan/full_scan.cu:96).
#include <cstdlib>

#include "common.cuh"
#include "internal.h"
#include "sched.cuh"

namespace fpscan {

// Pipeline depth and resident-CTA target, measured on B200 (forward, config
// 4 / config 5 sizes): fp32 with one vector per thread is fastest with an
// 8-deep ring at 3 CTAs/SM; half types with one vector per thread with 4
// stages at 4 CTAs/SM; two vectors per thread with 3 stages.
template <typename T, int NV>
struct FwdCfg {
  static constexpr bool kDeep = sizeof(T) == 4 && NV == 1;
  static constexpr int kStages = kDeep ? 8 : (NV == 1 ? 4 : (NV == 2 ? 3 : 2));
  static constexpr int kMinBlocks = kDeep ? 3 : 4;
  static constexpr int SV = kThreads * NV;  // 16-byte vectors per chunk
  static constexpr int smem_bytes() { return kStages * 2 * SV * 16; }
};

struct FwdKParams {
  const void* gates;
  const void* tokens;
  void* out;
  const float* init;
  float* carry_a;
  float* carry_b;
  int64_t rows;
  UnitSched us;  // rows per unit, units, counter (null: static, one unit per CTA)
  int lg;        // log2(seqlen)
  LinkParams lk;
};

// DIRECT: no shared-memory staging -- every thread loads its vectors from
// global memory itself.  Used for small launches whose rows fit in one
// chunk, where the staging pipeline's set-up (mbarrier init, one thread
// issuing the copies, waiting) is a visible share of a few-microsecond kernel.
//
// LINK (chained sequence sharding; multi-chunk rows, forward order only):
// bit 0 -- a row's initial state arrives from the upstream rank: at the row's
// first chunk thread 0 waits for the row's flag, reads the value, marks it
// consumed in the upstream rank's ack word and hands it to the CTA through
// shared memory; bit 1 -- the row's final state goes to the downstream rank
// (after its ack shows the ring slot free), released at system scope.
template <typename T, int NV, bool REV, bool HAS_OUT, bool HAS_INIT, bool HAS_CARRY_OUT,
          int ACT, bool DIRECT = false, int LINK = 0>
__global__ void __launch_bounds__(kThreads, (FwdCfg<T, NV>::kMinBlocks)) scan_fwd_kernel(const FwdKParams p) {
  constexpr int V = Elem<T>::kVec;   // elements per 16-byte vector
  constexpr int E = V * NV;          // elements per thread per chunk
  constexpr int CH = kThreads * E;   // elements per chunk
  constexpr int LGE = ilog2(E);
  constexpr int LGCH = ilog2(CH);
  constexpr int S = FwdCfg<T, NV>::kStages;
  constexpr int SV = FwdCfg<T, NV>::SV;

  extern __shared__ __align__(128) uint4 dsm[];
  uint4 (*s_g)[SV] = reinterpret_cast<uint4 (*)[SV]>(dsm);           // [S][SV]
  uint4 (*s_x)[SV] = reinterpret_cast<uint4 (*)[SV]>(dsm + S * SV);  // [S][SV]
  __shared__ __align__(8) uint64_t s_bar[S];
  __shared__ float2 s_wt[2][kWarps];
  __shared__ float s_link[2];  // LINK bit 0: the row's initial state, by chunk parity

  __shared__ int64_t s_abs[S];  // per stage: the chunk's first element in the tensor ...
  __shared__ int s_cnt[S];      // ... and its element count (0: end of work)
  __shared__ ProdState s_ps;

  const T* __restrict__ gates = static_cast<const T*>(p.gates);
  const T* __restrict__ tokens = static_cast<const T*>(p.tokens);
  T* out = static_cast<T*>(p.out);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int lg = p.lg;
  const int64_t Lmask = (int64_t(1) << lg) - 1;
  FPSCAN_DEBUG_ONLY(const int64_t n_el = p.rows << lg;)  // elements of each tensor
  if ((int64_t)blockIdx.x >= p.us.nunits) return;
  // Units are flat streams of whole rows (chunks never straddle units, and a
  // unit starts a row, so an element's position in its row is abs & Lmask).
  // Chunk positions reach the consumers through s_abs / s_cnt, except in
  // LOCAL variants (direct loads; links, which are always statically tiled),
  // where every thread computes them from its CTA's one tile.
  constexpr bool LOCAL = DIRECT;
  int64_t base0 = 0, n0 = 0, nck0 = 0;
  if constexpr (LOCAL) {
    const int64_t r0 = (int64_t)blockIdx.x * p.us.upr;
    base0 = r0 << lg;
    n0 = min(p.us.upr, p.rows - r0) << lg;
    nck0 = (n0 + CH - 1) >> LGCH;
  }

  const bool multi = lg > LGCH;                        // a row spans several chunks
  const int tpr = multi ? kThreads : 1 << (lg - LGE);  // threads per segment
  const int wwidth = tpr < 32 ? tpr : 32;
  const int seg_warps = tpr >> 5;

  if (!DIRECT) {
    if (tid == 0) {
#pragma unroll
      for (int s = 0; s < S; ++s) mbar_init(&s_bar[s], 1);
      fence_mbar_init();
    }
    __syncthreads();
  }
  // Everything above overlaps the previous kernel in the stream; from here
  // on global memory is touched.
  pdl_wait();
  pdl_launch_dependents();

  // Thread 0 fills the stages in order; after the last chunk of the last
  // unit it completes one more stage with no copy and count 0.
  unsigned claim = 0;
  auto issue_next = [&]() {
    ProdState& ps = s_ps;
    if (ps.done) return;
    const int s = (int)(ps.issued % S);
    ++ps.issued;
    if (ps.unit >= p.us.nunits) {
      ps.done = 1;
      s_cnt[s] = 0;
      mbar_arrive(&s_bar[s]);
      return;
    }
    const int64_t off = (REV ? ps.nck - 1 - ps.k : ps.k) << LGCH;
    const int64_t abs = ps.base + off;
    const int cnt = (int)min((int64_t)CH, ps.n - off);
    const uint32_t bytes = (uint32_t)cnt * (uint32_t)sizeof(T);
    s_abs[s] = abs;
    s_cnt[s] = cnt;
    // debug builds: a copy outside its tensor is skipped, the stage completes
    FPSCAN_DEBUG_ONLY(
        if (!in_bounds(gates + abs, bytes, gates, gates + n_el) ||
            !in_bounds(tokens + abs, bytes, tokens, tokens + n_el)) {
          mbar_arrive(&s_bar[s]);
        } else)
    {
      mbar_expect_tx(&s_bar[s], 2u * bytes);
      bulk_g2s(s_g[s], gates + abs, bytes, &s_bar[s]);
      bulk_g2s(s_x[s], tokens + abs, bytes, &s_bar[s]);
    }
    if (++ps.k == ps.nck) {
      ps.k = 0;
      prod_next_unit<CH>(ps, p.us, p.rows, lg, claim);
    }
  };
  if (!DIRECT && tid == 0) {
    prod_init<CH>(s_ps, p.us, p.rows, lg, claim);
    for (int i = 0; i < S; ++i) issue_next();
  }

  const int vi = REV ? kThreads - 1 - tid : tid;  // thread's slot (in NV-vector units)
  const int seg_lane_t = tid & (tpr - 1);          // thread index within its segment
  float carry = 0.f;  // state entering the current chunk (multi-chunk rows)
  float acc_a = 1.f;  // gate product of the current row so far (multi-chunk rows)
  int64_t k = 0;
  int s = 0;
  uint32_t phase = 0;
  bool aborted = false;

  for (;; ++k) {
    int64_t abs = 0;
    int cnt = 0;
    if constexpr (LOCAL) {
      if (k >= nck0) break;
      const int64_t off = (REV ? nck0 - 1 - k : k) << LGCH;
      abs = base0 + off;
      cnt = (int)min((int64_t)CH, n0 - off);
    }

    // LINK: start the polls this chunk needs (completed after pass 1).  The
    // polling thread is the producer, which wrote the stage's position
    // itself, so it may read it before the stage's copies land.
    uint64_t link_pre = 0;
    uint32_t ack_pre = 0;
    if constexpr (LINK != 0) {
      if (tid == 0 && s_cnt[s] != 0) {
        const int64_t pabs = s_abs[s];
        if ((LINK & 1) != 0 && multi && (pabs & Lmask) == 0)
          link_pre = ld_relaxed_sys_u64(p.lk.in_word + (pabs >> lg));
        if ((LINK & 2) != 0 && ((pabs + CH) & Lmask) == 0)
          ack_pre = ld_relaxed_sys_u32(p.lk.ack_in + (pabs >> lg));
      }
    }

    const bool ok = DIRECT || mbar_wait_bounded(&s_bar[s], phase);
    if constexpr (!LOCAL) {
      abs = s_abs[s];
      cnt = s_cnt[s];
    }
    const bool valid = (vi << LGE) < cnt;

    float a[E], b[E];
    if (valid) {
      Vec16<T> gv[NV], xv[NV];
      {
        uint4 rg[NV], rx[NV];
        if (DIRECT) {
          const uint4* gsrc = reinterpret_cast<const uint4*>(gates + abs) + vi * NV;
          const uint4* xsrc = reinterpret_cast<const uint4*>(tokens + abs) + vi * NV;
          FPSCAN_DEBUG_ONLY(
              const bool lok = in_bounds(gsrc, NV * 16, gates, gates + n_el) &&
                               in_bounds(xsrc, NV * 16, tokens, tokens + n_el);)
#pragma unroll
          for (int q = 0; q < NV; ++q) {
            FPSCAN_DEBUG_ONLY(if (!lok) { rg[q] = rx[q] = make_uint4(0, 0, 0, 0); continue; })
            rg[q] = __ldg(gsrc + q);
            rx[q] = __ldg(xsrc + q);
          }
        } else {
          lds_vecs<NV>(&s_g[s][vi * NV], rg);
          lds_vecs<NV>(&s_x[s][vi * NV], rx);
        }
#pragma unroll
        for (int q = 0; q < NV; ++q) {
          gv[q].raw = rg[q];
          xv[q].raw = rx[q];
        }
      }
#pragma unroll
      for (int i = 0; i < E; ++i) {
        const int j = REV ? E - 1 - i : i;
        const float g = act_fwd<ACT, T>(Elem<T>::load(gv[j / V].e[j % V]));
        const float x = Elem<T>::load(xv[j / V].e[j % V]);
        if (i == 0) {
          a[0] = g;
          b[0] = x;
        } else {
          a[i] = a[i - 1] * g;
          b[i] = fmaf(b[i - 1], g, x);
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < E; ++i) {
        a[i] = 1.f;
        b[i] = 0.f;
      }
    }

    float ta = a[E - 1], tb = b[E - 1], pa, pb;
    // Rows spanning whole chunks take the constant-width scans (no segment
    // arithmetic); short rows are scanned in segments of `wwidth` lanes.
    if (multi)
      warp_exclusive(ta, tb, lane, 32, pa, pb);
    else
      warp_exclusive(ta, tb, lane, wwidth, pa, pb);
    const int buf = (int)(k & 1);
    if (lane == 31) s_wt[buf][warp] = make_float2(ta, tb);
    if constexpr ((LINK & 1) != 0) {
      if (tid == 0 && multi && cnt != 0 && ((abs & Lmask) == 0)) {
        const int64_t lrow = abs >> lg;
        const float v = link_take(p.lk.in_word + lrow, p.lk.epoch, link_pre);
        s_link[buf] = v;
        if (p.lk.in_record) p.lk.in_record[lrow] = v;
        st_relaxed_sys_u32(p.lk.ack_out + lrow, p.lk.epoch);  // the slot may be reused
      }
    }

    if (__syncthreads_or(!ok)) {
      aborted = true;
      break;
    }
    if (cnt == 0) break;  // end-of-work marker
    // Every thread has consumed stage s: refill it.
    if (!DIRECT && tid == 0) issue_next();

    float ca = 1.f, cb = 0.f;
    if (multi)
      compose_warp_totals(s_wt[buf], lane, warp, kWarps, pa, pb, ca, cb);
    else if (seg_warps >= 2)
      compose_warp_totals(s_wt[buf], lane, warp, seg_warps, pa, pb, ca, cb);

    // Does this chunk start its row (in processing order)?
    const bool row_start = multi ? (((REV ? abs + CH : abs) & Lmask) == 0) : true;
    const int64_t row = (multi ? abs : abs + ((int64_t)vi << LGE)) >> lg;
    float state;  // y just before this thread's first element
    bool skip_state = false;
    if (row_start) {
      if (HAS_INIT) {
        carry = (LINK & 1) ? s_link[buf] : p.init[row];
        state = fmaf(pa, carry, pb);
      } else {
        carry = 0.f;
        state = pb;
        skip_state = seg_lane_t == 0;  // ignore the row's first gate
      }
    } else {
      state = fmaf(pa, carry, pb);
    }

    float yv[E];
#pragma unroll
    for (int i = 0; i < E; ++i) yv[i] = skip_state ? b[i] : fmaf(a[i], state, b[i]);

    if (HAS_OUT && valid) {
      float f[E];  // memory order
#pragma unroll
      for (int i = 0; i < E; ++i) f[REV ? E - 1 - i : i] = yv[i];
      uint4* dst = reinterpret_cast<uint4*>(out + abs) + vi * NV;
      FPSCAN_DEBUG_ONLY(if (in_bounds(dst, NV * 16, out, out + n_el)))
#pragma unroll
      for (int q = 0; q < NV; ++q) dst[q] = pack_vec<T>(f + q * V);
    }

    if (multi) {
      const float new_carry = (row_start && !HAS_INIT) ? cb : fmaf(ca, carry, cb);
      acc_a = (row_start ? 1.f : acc_a) * ca;
      carry = new_carry;
      if (HAS_CARRY_OUT && tid == 0 && ((REV ? abs : abs + CH) & Lmask) == 0
          FPSCAN_DEBUG_ONLY(&& in_bounds<4>(p.carry_a + row, 4, p.carry_a, p.carry_a + p.rows)
                            && in_bounds<4>(p.carry_b + row, 4, p.carry_b, p.carry_b + p.rows))) {
        p.carry_a[row] = acc_a;
        p.carry_b[row] = carry;
      }
      if constexpr ((LINK & 2) != 0) {
        if (tid == 0 && ((abs + CH) & Lmask) == 0) {
          // the slot's previous use (epoch - depth) must have been taken
          link_wait_ack(p.lk.ack_in + row, p.lk.epoch - p.lk.depth, ack_pre);
          st_relaxed_sys_u64(p.lk.out_word + row, link_word(carry, p.lk.epoch));
        }
      }
    } else if (HAS_CARRY_OUT && valid && seg_lane_t == tpr - 1
               FPSCAN_DEBUG_ONLY(&& in_bounds<4>(p.carry_a + row, 4, p.carry_a, p.carry_a + p.rows)
                                 && in_bounds<4>(p.carry_b + row, 4, p.carry_b, p.carry_b + p.rows))) {
      p.carry_a[row] = pa * a[E - 1];
      p.carry_b[row] = yv[E - 1];
    }

    if (++s == S) {
      s = 0;
      phase ^= 1u;
    }
  }

  if (aborted && tid == 0) {
    // Let copies already in flight land before the CTA's shared memory is
    // released, and make this CTA's remaining claims (its failing one
    // included) so the counter is still reset by the launch's last claim.
    for (int64_t kk = k; kk < s_ps.issued; ++kk)
      mbar_wait_bounded(&s_bar[kk % S], (uint32_t)((kk / S) & 1));
    drain_claims(s_ps.unit, p.us, claim);
  }
}

// One wave of CTAs (SMs x resident CTAs per SM, queried once per device and
// kernel).  With a unit counter and more units than CTAs, rows are handed out
// in units (plan_units); otherwise each CTA streams one contiguous tile.
template <typename T, int NV, bool REV, bool HAS_OUT, bool HAS_INIT, bool HAS_CARRY_OUT,
          int ACT, bool DIRECT = false, int LINK = 0>
static cudaError_t launch_fwd_t(const FwdArgs& a) {
  constexpr int smem = DIRECT ? 0 : FwdCfg<T, NV>::smem_bytes();
  auto kern = scan_fwd_kernel<T, NV, REV, HAS_OUT, HAS_INIT, HAS_CARRY_OUT, ACT, DIRECT, LINK>;
  static int occ_cache[64] = {0};
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
  const int64_t slots = (int64_t)a.num_sms * occ;
  constexpr int64_t kChunk = (int64_t)kThreads * Elem<T>::kVec * NV;
  // Links keep static tiles (every rank must tile its rows alike); direct
  // loads are for one-chunk tiles only.
  const UnitSched us = plan_units(a.rows, a.seqlen, kChunk, slots,
                                  (DIRECT || (LINK != 0 && !link_claims())) ? nullptr
                                                                            : a.sched);
  // Plain scans whose every tile is a single chunk (one wave of small
  // tiles) run the direct-load variant.
  if constexpr (!DIRECT && LINK == 0 && HAS_OUT && !HAS_INIT && !HAS_CARRY_OUT &&
                ACT == kActNone) {
    if (us.ctr == nullptr && us.upr * a.seqlen <= kChunk && !getenv("FPSCAN_B200_NO_DIRECT"))
      return launch_fwd_t<T, NV, REV, HAS_OUT, HAS_INIT, HAS_CARRY_OUT, ACT, true>(a);
  }
  UnitSched ul = us;
  if constexpr (DIRECT) {
    // Direct loads, short rows: pack as many rows per CTA as fill a chunk
    // (fewer, full CTAs) rather than one short row per CTA with most
    // threads idle.  Measured on BASELINE config 2 (512 rows, back-to-back
    // calls): L = 32 2.00 vs 2.41 us, L = 512 2.60 vs 2.75 us; at L = 1024
    // (two vectors per thread) 3.26 vs 3.16 us, so rows of 1024 and more
    // keep one row per CTA.  FPSCAN_B200_DIRECT_PACK=0 keeps the one-wave
    // tiling everywhere.
    static const bool pack = [] {
      const char* v = getenv("FPSCAN_B200_DIRECT_PACK");
      return !(v && v[0] == '0');
    }();
    if (pack && a.seqlen <= 512 && a.seqlen < kChunk && ul.upr * a.seqlen < kChunk) {
      ul.upr = kChunk / a.seqlen;
      ul.nunits = (a.rows + ul.upr - 1) / ul.upr;
      ul.grid = ul.nunits;
    }
  }
  FwdKParams p{a.gates, a.tokens, a.out, a.init, a.carry_a, a.carry_b, a.rows, ul,
               ilog2_host(a.seqlen), a.lk};
  return launch_pdl(kern, (unsigned)ul.grid, kThreads, smem, a.stream, p);
}

template <typename T, bool REV, bool HAS_OUT, bool HAS_INIT, bool HAS_CARRY_OUT, int ACT = kActNone>
static cudaError_t launch_fwd_nv(const FwdArgs& a) {
  if constexpr (sizeof(T) == 4 && ACT == kActNone)
    if (a.nv == 4) return launch_fwd_t<T, 4, REV, HAS_OUT, HAS_INIT, HAS_CARRY_OUT, ACT>(a);
  return a.nv == 1 ? launch_fwd_t<T, 1, REV, HAS_OUT, HAS_INIT, HAS_CARRY_OUT, ACT>(a)
                   : launch_fwd_t<T, 2, REV, HAS_OUT, HAS_INIT, HAS_CARRY_OUT, ACT>(a);
}

template <typename T, bool REV>
static cudaError_t launch_fwd_act(const FwdArgs& a) {
  switch (a.act) {
    case kActSigmoid:
      return launch_fwd_nv<T, REV, true, false, false, kActSigmoid>(a);
    case kActExpNegSoftplus:
      return launch_fwd_nv<T, REV, true, false, false, kActExpNegSoftplus>(a);
    case kActExp:
      return launch_fwd_nv<T, REV, true, false, false, kActExp>(a);
    default:
      return launch_fwd_nv<T, REV, true, false, false>(a);
  }
}

// Chained sequence sharding: link bit 0 (init from upstream) implies
// HAS_INIT; one or two vectors per thread.
template <typename T, int LINK>
static cudaError_t launch_fwd_link_t(const FwdArgs& a) {
  constexpr bool kInit = (LINK & 1) != 0;
  return a.nv == 1 ? launch_fwd_t<T, 1, false, true, kInit, false, kActNone, false, LINK>(a)
                   : launch_fwd_t<T, 2, false, true, kInit, false, kActNone, false, LINK>(a);
}

template <typename T>
static cudaError_t launch_fwd_dtype(const FwdArgs& a) {
  if (a.link != 0) {
    if (a.reverse || a.act != kActNone || a.carry_a != nullptr || a.out == nullptr)
      return cudaErrorInvalidValue;
    switch (a.link) {
      case 1:
        return launch_fwd_link_t<T, 1>(a);
      case 2:
        return launch_fwd_link_t<T, 2>(a);
      case 3:
        return launch_fwd_link_t<T, 3>(a);
      default:
        return cudaErrorInvalidValue;
    }
  }
  const bool has_out = a.out != nullptr;
  const bool has_init = a.init != nullptr;
  const bool has_co = a.carry_a != nullptr;
  // Instantiated variants: plain scan (fwd/rev); forward with init
  // (+carry-out); carry-out only (reduce).
  if (has_out && !has_init && !has_co)
    return a.reverse ? launch_fwd_act<T, true>(a) : launch_fwd_act<T, false>(a);
  if (a.act != kActNone) return cudaErrorInvalidValue;
  if (has_out && has_init && !has_co)
    return a.reverse ? launch_fwd_nv<T, true, true, true, false>(a)
                     : launch_fwd_nv<T, false, true, true, false>(a);
  if (a.reverse) return cudaErrorInvalidValue;
  if (has_out && has_init && has_co) return launch_fwd_nv<T, false, true, true, true>(a);
  if (has_out && !has_init && has_co) return launch_fwd_nv<T, false, true, false, true>(a);
  if (!has_out && !has_init && has_co) return launch_fwd_nv<T, false, false, false, true>(a);
  return cudaErrorInvalidValue;
}

cudaError_t launch_fwd(const FwdArgs& a) {
  switch (a.dtype) {
    case kF32:
      return launch_fwd_dtype<float>(a);
    case kF16:
      return launch_fwd_dtype<__half>(a);
    case kBF16:
      return launch_fwd_dtype<__nv_bfloat16>(a);
    default:
      return cudaErrorInvalidValue;
  }
}

}  // namespace fpscan
