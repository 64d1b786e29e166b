// Fused backward of the linear-recurrence scan, sm_100a.
//
// The reference composes PScan.backward from five launches
// (fpscan/ops.py:70-83): shift the gates left (torch.cat + slice +
// contiguous), a reverse scan_forward of grad_out over the shifted gates, shift
// y right (torch.cat + slice) and a multiply:
//     dtokens[t] = gates[t+1] * dtokens[t+1] + grad_out[t]   (t = L-1: no term)
//     dgates[t]  = dtokens[t] * y[t-1]                         (y[-1] = 0)
// Here one kernel does all of it in a single reverse pass: it reads gates,
// grad_out and y once (3 reads) and writes dgates and dtokens (2 writes).
// The one-element shifts are served from the staged chunks: the gates stage
// carries one extra 16-byte vector after the chunk, the y stage one before it,
// so no global re-reads are needed for the halos.
//
// Pipeline, row-unit scheduling, segmentation of short rows and carry
// handling follow scan_fwd.cu.  The thread-level scan is two-pass: a thread
// folds its group into one map before the block scan and re-runs the
// recurrence from the entering state after it, so no per-element results
// are live across the barrier (only the inputs: packed, or for half types at
// one vector per thread their fp32 conversions, which pass 2 reuses).  Optional per-row `addend` (value entering at the row's last
// element, i.e. gates[L] * dtokens[L] of the next sequence shard) and
// `y_prev` (y before the row's first element, from the previous shard) serve
// the sequence-sharded mode; reduce mode (no outputs) emits per row
// gates[0] * dtokens[0], the value the previous shard needs.
#include "common.cuh"
#include "internal.h"
#include "sched.cuh"

namespace fpscan {

template <int NV>
struct BwdCfg {
  static constexpr int kStages = NV == 1 ? 4 : (NV == 2 ? 3 : 2);
  static constexpr int kMinBlocks = NV == 4 ? 2 : 3;  // resident CTAs the smem ring allows
  static constexpr int SV = kThreads * NV;  // 16-byte vectors per chunk
  static constexpr int GS = SV + 1;         // gates stage: chunk + one vector after
  static constexpr int YS = SV + 1;         // y stage: one vector before + chunk
  template <bool HAS_OUT>
  static constexpr int smem_bytes() {
    return kStages * 16 * (GS + SV + (HAS_OUT ? YS : 0));
  }
};

struct BwdKParams {
  const void* gates;
  const void* y;
  const void* gout;
  void* dgates;
  void* dtok;
  const float* addend;
  const float* y_prev;
  float* carry_b;
  int64_t rows;
  UnitSched us;  // rows per unit, units, counter (null: static, one unit per CTA)
  int lg;
  LinkParams lk;
};

// LINK (chained sequence sharding; multi-chunk rows): bit 0 -- the value
// entering a row's last element (the downstream rank's gates[0]*dtokens[0])
// arrives over the link (thread 0 waits, reads, acks, shares through shared
// memory); bit 1 -- this rank's gates[0]*dtokens[0] of each row goes to the
// upstream rank.  Link kernels always take y[-1] of each row from y_prev.
// Half types at one vector per thread keep their fp32 inputs across the
// barrier; the bound of 4 CTAs per SM holds them at <= 64 registers (62, no
// spills), where the 4-stage ring also fits 4 CTAs.
template <typename T, int NV, int ACT>
constexpr int bwd_min_blocks() {
  return (sizeof(T) == 2 && NV == 1 && ACT == kActNone) ? 4 : BwdCfg<NV>::kMinBlocks;
}

template <typename T, int NV, bool HAS_OUT, bool HAS_CARRY, int ACT, int LINK = 0>
__global__ void __launch_bounds__(kThreads, (bwd_min_blocks<T, NV, ACT>()))
    scan_bwd_kernel(const BwdKParams p) {
  constexpr int V = Elem<T>::kVec;
  constexpr int E = V * NV;
  constexpr int CH = kThreads * E;
  constexpr int LGE = ilog2(E);
  constexpr int LGCH = ilog2(CH);
  using Cfg = BwdCfg<NV>;
  constexpr int S = Cfg::kStages;
  constexpr int SV = Cfg::SV, GS = Cfg::GS, YS = Cfg::YS;

  extern __shared__ __align__(128) uint4 dsm[];
  uint4* s_g = dsm;               // [S][GS]
  uint4* s_go = s_g + S * GS;     // [S][SV]
  uint4* s_y = s_go + S * SV;     // [S][YS]   (HAS_OUT only)
  __shared__ __align__(8) uint64_t s_bar[S];
  __shared__ float2 s_wt[2][kWarps];
  __shared__ float s_link[2];  // LINK bit 0: value entering the row, by chunk parity

  const T* __restrict__ gates = static_cast<const T*>(p.gates);
  const T* __restrict__ y = static_cast<const T*>(p.y);
  const T* __restrict__ gout = static_cast<const T*>(p.gout);
  T* __restrict__ dgates = static_cast<T*>(p.dgates);
  T* __restrict__ dtok = static_cast<T*>(p.dtok);

  __shared__ int64_t s_abs[S];  // per stage: the chunk's first element in the tensor ...
  __shared__ int s_cnt[S];      // ... and its element count (0: end of work)
  __shared__ ProdState s_ps;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int lg = p.lg;
  const int64_t Lmask = (int64_t(1) << lg) - 1;
  FPSCAN_DEBUG_ONLY(const int64_t n_el = p.rows << lg;)  // elements of each tensor
  if ((int64_t)blockIdx.x >= p.us.nunits) return;
  // Units and chunk hand-over as in scan_fwd.cu; link variants (always
  // statically tiled) compute their chunk positions in every thread.
  constexpr bool LOCAL = false;
  int64_t base0 = 0, n0 = 0, nck0 = 0;
  if constexpr (LOCAL) {
    const int64_t r0 = (int64_t)blockIdx.x * p.us.upr;
    base0 = r0 << lg;
    n0 = min(p.us.upr, p.rows - r0) << lg;
    nck0 = (n0 + CH - 1) >> LGCH;
  }

  const bool multi = lg > LGCH;
  const int tpr = multi ? kThreads : 1 << (lg - LGE);
  const int wwidth = tpr < 32 ? tpr : 32;
  const int seg_warps = tpr >> 5;

  if (tid == 0) {
#pragma unroll
    for (int s = 0; s < S; ++s) mbar_init(&s_bar[s], 1);
    fence_mbar_init();
  }
  __syncthreads();
  // Everything above overlaps the previous kernel in the stream; from here
  // on global memory is touched.
  pdl_wait();
  pdl_launch_dependents();

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
    const int64_t off = (ps.nck - 1 - ps.k) << LGCH;  // reverse processing order
    const int64_t abs = ps.base + off;
    const int cnt = (int)min((int64_t)CH, ps.n - off);
    const uint32_t bytes = (uint32_t)cnt * (uint32_t)sizeof(T);
    // halos within the unit: the gate after the chunk, the y before it
    const uint32_t g_bytes = bytes + ((off + cnt < ps.n) ? 16u : 0u);
    uint32_t y_bytes = 0;
    if (HAS_OUT) y_bytes = bytes + (off > 0 ? 16u : 0u);
    s_abs[s] = abs;
    s_cnt[s] = cnt;
    // debug builds: a copy outside its tensor is skipped, the stage completes
    FPSCAN_DEBUG_ONLY(
        if (!in_bounds(gates + abs, g_bytes, gates, gates + n_el) ||
            !in_bounds(gout + abs, bytes, gout, gout + n_el) ||
            (HAS_OUT && !in_bounds(off > 0 ? y + abs - V : y + abs, y_bytes, y, y + n_el))) {
          mbar_arrive(&s_bar[s]);
        } else)
    {
      mbar_expect_tx(&s_bar[s], g_bytes + bytes + y_bytes);
      bulk_g2s(s_g + s * GS, gates + abs, g_bytes, &s_bar[s]);
      bulk_g2s(s_go + s * SV, gout + abs, bytes, &s_bar[s]);
      if (HAS_OUT) {
        if (off > 0)
          bulk_g2s(s_y + s * YS, y + abs - V, y_bytes, &s_bar[s]);
        else
          bulk_g2s(s_y + s * YS + 1, y + abs, y_bytes, &s_bar[s]);
      }
    }
    if (++ps.k == ps.nck) {
      ps.k = 0;
      prod_next_unit<CH>(ps, p.us, p.rows, lg, claim);
    }
  };
  if (tid == 0) {
    prod_init<CH>(s_ps, p.us, p.rows, lg, claim);
    for (int i = 0; i < S; ++i) issue_next();
  }

  const int vi = kThreads - 1 - tid;  // slot in NV-vector units, reverse order
  const int seg_lane_t = tid & (tpr - 1);
  float carry = 0.f;
  int64_t k = 0;
  int s = 0;
  uint32_t phase = 0;
  bool aborted = false;

  for (;; ++k) {
    int64_t abs = 0;
    int cnt = 0;
    if constexpr (LOCAL) {
      if (k >= nck0) break;
      const int64_t off = (nck0 - 1 - k) << LGCH;
      abs = base0 + off;
      cnt = (int)min((int64_t)CH, n0 - off);
    }

    // LINK: start the polls this chunk needs (completed after pass 1)
    // (the polling thread of bit 0 is the producer, which wrote the stage's
    // position itself; the ack words of bit 1 are read by the threads that
    // hold a row's first element, once the stage's position is visible)
    uint64_t link_pre = 0;
    uint32_t ack_pre = 0;
    if constexpr ((LINK & 1) != 0) {
      if (tid == 0 && s_cnt[s] != 0) {
        const int64_t pabs = s_abs[s];
        if (multi && ((pabs + CH) & Lmask) == 0)
          link_pre = ld_relaxed_sys_u64(p.lk.in_word + (pabs >> lg));
      }
    }

    const bool ok = mbar_wait_bounded(&s_bar[s], phase);
    if constexpr (!LOCAL) {
      abs = s_abs[s];
      cnt = s_cnt[s];
    }
    if constexpr ((LINK & 2) != 0) {
      const int64_t vs = abs + ((int64_t)vi << LGE);
      if ((vi << LGE) < cnt && (vs & Lmask) == 0)
        ack_pre = ld_relaxed_sys_u32(p.lk.ack_in + (vs >> lg));
    }
    const int64_t vstart = abs + ((int64_t)vi << LGE);  // thread's first element
    // Rows longer than a chunk come in whole chunks (cnt == CH, or 0 for the
    // end marker, whose pass 1 is discarded).  Row flags need only the low
    // 32 bits of the position (seqlen <= 2^24).
    const bool valid = multi || (vi << LGE) < cnt;
    const uint32_t vlo = (uint32_t)abs + ((uint32_t)vi << LGE);
    const uint32_t lmask = (uint32_t)Lmask;
    const bool grp_row_end = ((vlo + E) & lmask) == 0;  // holds a row's last element
    const bool grp_row_first = (vlo & lmask) == 0;      // holds a row's first element

    Vec16<T> gv[NV], gov[NV], yv[NV];
    float g_next = 1.f, y_before = 0.f;
    // Two passes over the inputs: fold the thread's elements into its map
    // (ta, tb) now, re-run the recurrence from the entering state after the
    // block scan (no per-element results live across the barrier).
    float ta = 1.f, tb = 0.f;
    {
      // Halo elements: gates[vstart+E] (first gate of the next slot) and
      // y[vstart-1] (last y of the previous slot).
      uint4 rg[NV], rgo[NV], ry[NV];
      const uint4* sg = s_g + s * GS + vi * NV;
      const uint4* sy = s_y + s * YS + 1 + vi * NV;
      if (valid) {
        lds_vecs<NV>(sg, rg);
        lds_vecs<NV>(s_go + s * SV + vi * NV, rgo);
        if (HAS_OUT) lds_vecs<NV>(sy, ry);
      } else {
#pragma unroll
        for (int q = 0; q < NV; ++q) rg[q] = rgo[q] = ry[q] = make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int q = 0; q < NV; ++q) {
        gv[q].raw = rg[q];
        gov[q].raw = rgo[q];
        if (HAS_OUT) yv[q].raw = ry[q];
      }
      if (valid && !grp_row_end)
        g_next = act_fwd<ACT, T>(Elem<T>::load(reinterpret_cast<const T*>(sg + NV)[0]));
      if (HAS_OUT && valid && !grp_row_first)
        y_before = Elem<T>::load(reinterpret_cast<const T*>(sy)[-1]);
    }
    // Half types, one vector, no activation: the converted gates and
    // grad_out stay in registers for pass 2 instead of the packed vectors.
    constexpr bool kKeepF = sizeof(T) == 2 && NV == 1 && ACT == kActNone;
    float cg[kKeepF ? E : 1], cx[kKeepF ? E : 1];
    if constexpr (kKeepF) {
#pragma unroll
      for (int j = 0; j < E; ++j) {
        cg[j] = Elem<T>::load(gv[j / V].e[j % V]);
        cx[j] = Elem<T>::load(gov[j / V].e[j % V]);
      }
    }
    if (valid) {
#pragma unroll
      for (int i = 0; i < E; ++i) {
        const int j = E - 1 - i;  // element within the thread's group, memory order
        float g, x;
        if constexpr (kKeepF) {
          g = (j == E - 1) ? g_next : cg[j + 1];
          x = cx[j];
        } else {
          g = (j == E - 1) ? g_next
                           : act_fwd<ACT, T>(Elem<T>::load(gv[(j + 1) / V].e[(j + 1) % V]));
          x = Elem<T>::load(gov[j / V].e[j % V]);
        }
        ta = i == 0 ? g : ta * g;
        tb = i == 0 ? x : fmaf(tb, g, x);
      }
    }

    float pa, pb;
    // rows longer than a chunk (the common case): full-warp segments, the
    // widths fixed at compile time
    if (multi)
      warp_exclusive(ta, tb, lane, 32, pa, pb);
    else
      warp_exclusive(ta, tb, lane, wwidth, pa, pb);
    const int buf = (int)(k & 1);
    if (lane == 31) s_wt[buf][warp] = make_float2(ta, tb);
    if constexpr ((LINK & 1) != 0) {
      if (tid == 0 && multi && cnt != 0 && (((abs + CH) & Lmask) == 0)) {
        const int64_t lrow = abs >> lg;
        s_link[buf] = link_take(p.lk.in_word + lrow, p.lk.epoch, link_pre);
        st_relaxed_sys_u32(p.lk.ack_out + lrow, p.lk.epoch);  // the slot may be reused
      }
    }

    if (__syncthreads_or(!ok)) {
      aborted = true;
      break;
    }
    if (cnt == 0) break;  // end-of-work marker
    if (tid == 0) issue_next();

    float ca = 1.f, cb = 0.f;
    if (multi)
      compose_warp_totals(s_wt[buf], lane, warp, kWarps, pa, pb, ca, cb);
    else if (seg_warps >= 2)
      compose_warp_totals(s_wt[buf], lane, warp, seg_warps, pa, pb, ca, cb);

    const bool row_start = multi ? ((((uint32_t)abs + CH) & lmask) == 0) : true;  // processing order
    const int64_t row = (multi ? abs : vstart) >> lg;
    float state;
    bool skip_state = false;
    if (row_start) {
      if (HAS_CARRY) {
        carry = (LINK & 1) ? s_link[buf] : p.addend[row];
        state = fmaf(pa, carry, pb);
      } else {
        carry = 0.f;
        state = pb;
        skip_state = seg_lane_t == 0;
      }
    } else {
      state = fmaf(pa, carry, pb);
    }

    // Pass 2, in processing order (element j = E-1-i at step i): dtokens by
    // the recurrence from `state`, and dgates.  Each element's activated
    // gate serves its own gradient factor and the next step's recurrence, so
    // the activation is evaluated once per element here (once in pass 1).
    float yp_first = y_before;
    if (HAS_OUT && valid && grp_row_first)
      yp_first = (HAS_CARRY || LINK != 0) ? p.y_prev[row] : 0.f;
    float d = state;
    float gcur = g_next;  // activated gate of element j + 1
    // Each 16-byte vector is packed and stored as soon as its elements are
    // done, so only one vector's results are live at a time.
    uint4* d1 = HAS_OUT ? reinterpret_cast<uint4*>(dtok + abs) + vi * NV : nullptr;
    uint4* d2 = HAS_OUT ? reinterpret_cast<uint4*>(dgates + abs) + vi * NV : nullptr;
    bool st_ok = valid;
    FPSCAN_DEBUG_ONLY(if (HAS_OUT) st_ok = st_ok && in_bounds(d1, NV * 16, dtok, dtok + n_el) &&
                                           in_bounds(d2, NV * 16, dgates, dgates + n_el);)
#pragma unroll
    for (int qq = 0; qq < NV; ++qq) {
      const int q = NV - 1 - qq;
      float f_dt[HAS_OUT ? V : 1], f_dg[HAS_OUT ? V : 1];  // memory order within the vector
#pragma unroll
      for (int ii = 0; ii < V; ++ii) {
        const int i = qq * V + ii;
        const int jv = V - 1 - ii;
        const int j = q * V + jv;
        float x, gj;
        if constexpr (kKeepF) {
          x = cx[j];
          gj = cg[j];
        } else {
          x = Elem<T>::load(gov[q].e[jv]);
          gj = act_fwd<ACT, T>(Elem<T>::load(gv[q].e[jv]));
        }
        d = (i == 0 && skip_state) ? x : fmaf(gcur, d, x);
        if constexpr (HAS_OUT) {
          const float yp = (j == 0) ? yp_first : Elem<T>::load(yv[(j - 1) / V].e[(j - 1) % V]);
          f_dt[jv] = d;
          if constexpr (ACT == kActNone)
            f_dg[jv] = d * yp;
          else
            f_dg[jv] = d * yp * act_grad<ACT>(gj);
        }
        gcur = gj;
      }
      if constexpr (HAS_OUT) {
        if (st_ok) {
          d1[q] = pack_vec<T>(f_dt);
          d2[q] = pack_vec<T>(f_dg);
        }
      }
    }
    // now d = dtokens of the group's first element, gcur = its (activated) gate

    if (valid) {
      if constexpr (HAS_OUT) {
        if constexpr ((LINK & 2) != 0) {
          if (grp_row_first) {
            const float v = gcur * d;
            // the slot's previous use (epoch - depth) must have been taken
            link_wait_ack(p.lk.ack_in + row, p.lk.epoch - p.lk.depth, ack_pre);
            st_relaxed_sys_u64(p.lk.out_word + row, link_word(v, p.lk.epoch));
          }
        }
      } else if (grp_row_first FPSCAN_DEBUG_ONLY(
                     && in_bounds<4>(p.carry_b + row, 4, p.carry_b, p.carry_b + p.rows))) {
        p.carry_b[row] = gcur * d;  // plain scan only
      }
    }

    if (multi) carry = (row_start && !HAS_CARRY) ? cb : fmaf(ca, carry, cb);

    if (++s == S) {
      s = 0;
      phase ^= 1u;
    }
  }

  if (aborted && tid == 0) {
    // in-flight copies land first; remaining claims keep the counter's reset
    for (int64_t kk = k; kk < s_ps.issued; ++kk)
      mbar_wait_bounded(&s_bar[kk % S], (uint32_t)((kk / S) & 1));
    drain_claims(s_ps.unit, p.us, claim);
  }
}

template <typename T, int NV, bool HAS_OUT, bool HAS_CARRY, int ACT, int LINK = 0>
static cudaError_t launch_bwd_t(const BwdArgs& a) {
  constexpr int smem = BwdCfg<NV>::template smem_bytes<HAS_OUT>();
  auto kern = scan_bwd_kernel<T, NV, HAS_OUT, HAS_CARRY, ACT, LINK>;
  // Per device: opt in to >48 KiB of dynamic shared memory and cache the
  // number of resident CTAs.
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
  const UnitSched us =
      plan_units(a.rows, a.seqlen, kChunk, slots,
                 (LINK != 0 && !link_claims()) ? nullptr : a.sched);
  BwdKParams p{a.gates, a.y, a.grad_out, a.dgates, a.dtokens, a.addend, a.y_prev, a.carry_b,
               a.rows, us, ilog2_host(a.seqlen), a.lk};
  return launch_pdl(kern, (unsigned)us.grid, kThreads, smem, a.stream, p);
}

template <typename T, bool HAS_OUT, bool HAS_CARRY, int ACT = kActNone>
static cudaError_t launch_bwd_nv(const BwdArgs& a) {
  if constexpr (sizeof(T) == 4 && ACT == kActNone)
    if (a.nv == 4) return launch_bwd_t<T, 4, HAS_OUT, HAS_CARRY, ACT>(a);
  return a.nv == 1 ? launch_bwd_t<T, 1, HAS_OUT, HAS_CARRY, ACT>(a)
                   : launch_bwd_t<T, 2, HAS_OUT, HAS_CARRY, ACT>(a);
}

// Chained sequence sharding: link bit 0 (value entering from downstream)
// implies HAS_CARRY; one or two vectors per thread.
template <typename T, int LINK>
static cudaError_t launch_bwd_link_t(const BwdArgs& a) {
  constexpr bool kCarry = (LINK & 1) != 0;
  return a.nv == 1 ? launch_bwd_t<T, 1, true, kCarry, kActNone, LINK>(a)
                   : launch_bwd_t<T, 2, true, kCarry, kActNone, LINK>(a);
}

template <typename T>
static cudaError_t launch_bwd_dtype(const BwdArgs& a) {
  if (a.link != 0) {
    if (a.act != kActNone || a.dtokens == nullptr || a.y_prev == nullptr)
      return cudaErrorInvalidValue;
    switch (a.link) {
      case 1:
        return launch_bwd_link_t<T, 1>(a);
      case 2:
        return launch_bwd_link_t<T, 2>(a);
      case 3:
        return launch_bwd_link_t<T, 3>(a);
      default:
        return cudaErrorInvalidValue;
    }
  }
  const bool has_out = a.dtokens != nullptr;
  const bool has_carry = a.addend != nullptr;
  if (has_out && !has_carry) {
    switch (a.act) {
      case kActSigmoid:
        return launch_bwd_nv<T, true, false, kActSigmoid>(a);
      case kActExpNegSoftplus:
        return launch_bwd_nv<T, true, false, kActExpNegSoftplus>(a);
      case kActExp:
        return launch_bwd_nv<T, true, false, kActExp>(a);
      default:
        return launch_bwd_nv<T, true, false>(a);
    }
  }
  if (a.act != kActNone) return cudaErrorInvalidValue;
  if (has_out) return launch_bwd_nv<T, true, true>(a);
  return launch_bwd_nv<T, false, false>(a);
}

cudaError_t launch_bwd(const BwdArgs& a) {
  switch (a.dtype) {
    case kF32:
      return launch_bwd_dtype<float>(a);
    case kF16:
      return launch_bwd_dtype<__half>(a);
    case kBF16:
      return launch_bwd_dtype<__nv_bfloat16>(a);
    default:
      return cudaErrorInvalidValue;
  }
}

}  // namespace fpscan
