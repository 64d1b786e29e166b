// Forward / reverse linear-recurrence scan over the last axis of a
// (rows, L) row-major tensor, sm_100a.
//
// Replaces the reference kernel scan<> (csrc/full_scan/full_scan.cu:50-177)
// with a different design:
//   * one CTA streams a tile of whole rows, chunk by chunk (4 KiB per tensor
//     per chunk), through a kStages-deep shared-memory ring filled by
//     non-multicast cp.async.bulk copies completing on mbarriers, so several
//     chunks per CTA are in flight while the current one is scanned;
//   * per-thread serial scan over one 16-byte vector (4 fp32 / 8 half),
//     warp-shuffle Hillis-Steele scan of the thread totals, then a
//     per-warp redundant composition of the (double-buffered) warp totals --
//     one __syncthreads per chunk;
//   * rows shorter than a chunk are packed several to a chunk and scanned as
//     independent segments (row boundaries coincide with power-of-two thread
//     groups), rows longer than a chunk carry their fp32 state across chunks;
//   * 64-bit offsets throughout; any number of rows (no gridDim.y limit).
// Optional per-row initial state (`init`) and per-row carry-out
// (A = product of all gates of the row, B = final state) serve the
// sequence-sharded multi-GPU mode.  Without `init` the gate of a row's first
// element is ignored, exactly like the reference's forced 1.0
// (csrc/full_scan/full_scan.cu:96).
#include "common.cuh"
#include "internal.h"

namespace fpscan {

constexpr int kFwdStages = 4;

template <typename T, bool REV, bool HAS_OUT, bool HAS_INIT, bool HAS_CARRY_OUT>
__global__ void __launch_bounds__(kThreads)
    scan_fwd_kernel(const T* __restrict__ gates, const T* __restrict__ tokens, T* out,
                    const float* __restrict__ init, float* __restrict__ carry_a,
                    float* __restrict__ carry_b, int64_t rows, int64_t L,
                    int64_t rows_per_tile) {
  constexpr int V = Elem<T>::kVec;
  constexpr int CH = kThreads * V;  // elements per chunk
  constexpr int S = kFwdStages;

  __shared__ __align__(128) uint4 s_g[S][kThreads];
  __shared__ __align__(128) uint4 s_x[S][kThreads];
  __shared__ __align__(8) uint64_t s_bar[S];
  __shared__ float s_wa[2][kWarps], s_wb[2][kWarps];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t row0 = (int64_t)blockIdx.x * rows_per_tile;
  const int64_t nrows = min(rows_per_tile, rows - row0);
  const int64_t base = row0 * L;
  const int64_t n = nrows * L;
  const int64_t nck = (n + CH - 1) / CH;

  const bool multi = L > CH;  // a row spans several chunks
  const int tpr = multi ? kThreads : (int)(L / V);  // threads per segment (power of two)
  const int wwidth = tpr < 32 ? tpr : 32;
  const int seg_warps = tpr >> 5;  // warps per segment, 0 if sub-warp

  if (tid == 0) {
#pragma unroll
    for (int s = 0; s < S; ++s) mbar_init(&s_bar[s], 1);
    fence_mbar_init();
  }
  __syncthreads();

  int64_t issued = 0;  // meaningful in thread 0 only
  auto issue = [&](int64_t k) {
    const int64_t mc = REV ? nck - 1 - k : k;
    const int64_t off = mc * CH;
    const int64_t cnt = min((int64_t)CH, n - off);
    const uint32_t bytes = (uint32_t)(cnt * (int64_t)sizeof(T));
    const int s = (int)(k % S);
    mbar_expect_tx(&s_bar[s], 2u * bytes);
    bulk_g2s(s_g[s], gates + base + off, bytes, &s_bar[s]);
    bulk_g2s(s_x[s], tokens + base + off, bytes, &s_bar[s]);
  };
  if (tid == 0) {
    for (; issued < min((int64_t)S, nck); ++issued) issue(issued);
  }

  const int vi = REV ? kThreads - 1 - tid : tid;  // vector slot in the chunk
  const int seg_lane_t = tid & (tpr - 1);          // thread index in its segment
  float carry = 0.f;  // state entering the current chunk (multi-chunk rows)
  float acc_a = 1.f;  // running gate product of the current row (multi-chunk rows)
  int64_t k = 0;
  bool aborted = false;

  for (; k < nck; ++k) {
    const int s = (int)(k % S);
    const uint32_t parity = (uint32_t)((k / S) & 1);
    const int64_t mc = REV ? nck - 1 - k : k;
    const int64_t off = mc * CH;
    const int64_t cnt = min((int64_t)CH, n - off);
    const bool valid = (int64_t)vi * V < cnt;

    const bool ok = mbar_wait_bounded(&s_bar[s], parity);

    float a[V], b[V];
    if (valid) {
      Vec16<T> gv, xv;
      gv.raw = s_g[s][vi];
      xv.raw = s_x[s][vi];
#pragma unroll
      for (int i = 0; i < V; ++i) {
        const int j = REV ? V - 1 - i : i;
        const float g = Elem<T>::load(gv.e[j]);
        const float x = Elem<T>::load(xv.e[j]);
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
      for (int i = 0; i < V; ++i) {
        a[i] = 1.f;
        b[i] = 0.f;
      }
    }

    // Inclusive scan of thread totals within the warp segment, then the
    // exclusive prefix of this thread.
    float ta = a[V - 1], tb = b[V - 1];
    warp_scan_pair(ta, tb, lane, wwidth);
    float ea = __shfl_up_sync(0xffffffffu, ta, 1);
    float eb = __shfl_up_sync(0xffffffffu, tb, 1);
    if ((lane & (wwidth - 1)) == 0) {
      ea = 1.f;
      eb = 0.f;
    }
    const int wb_buf = (int)(k & 1);
    if (lane == 31) {
      s_wa[wb_buf][warp] = ta;
      s_wb[wb_buf][warp] = tb;
    }
    if (__syncthreads_or(!ok)) {
      aborted = true;
      break;
    }
    // Every thread has consumed stage s: refill it.
    if (tid == 0 && issued < nck) {
      issue(issued);
      ++issued;
    }

    // Prefix of the warps before this one in the segment, and (multi-chunk
    // rows) the composition of the whole chunk.
    float wa = 1.f, wbv = 0.f, ca = 1.f, cb = 0.f;
    if (seg_warps >= 2) {
      const int first = warp & ~(seg_warps - 1);
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        const float A = s_wa[wb_buf][w], B = s_wb[wb_buf][w];
        if (w >= first && w < warp) {
          wbv = fmaf(wbv, A, B);
          wa *= A;
        }
        cb = fmaf(cb, A, B);
        ca *= A;
      }
    }
    const float pa = wa * ea;
    const float pb = fmaf(wbv, ea, eb);

    // Does this chunk start its row (in processing order)?
    const bool row_start = multi ? (((REV ? off + CH : off) % L) == 0) : true;
    const int64_t row = row0 + (multi ? off : off + (int64_t)vi * V) / L;
    float state;  // y just before this thread's first element
    bool skip_state = false;
    if (row_start) {
      if (HAS_INIT) {
        carry = init[row];
        state = fmaf(pa, carry, pb);
      } else {
        carry = 0.f;
        state = pb;
        skip_state = seg_lane_t == 0;  // ignore the row's first gate
      }
    } else {
      state = fmaf(pa, carry, pb);
    }

    float yv[V];
#pragma unroll
    for (int i = 0; i < V; ++i) yv[i] = skip_state ? b[i] : fmaf(a[i], state, b[i]);

    if (HAS_OUT && valid) {
      Vec16<T> ov;
#pragma unroll
      for (int i = 0; i < V; ++i) ov.e[REV ? V - 1 - i : i] = Elem<T>::store(yv[i]);
      reinterpret_cast<uint4*>(out + base + off)[vi] = ov.raw;
    }

    if (multi) {
      const float new_carry = (row_start && !HAS_INIT) ? cb : fmaf(ca, carry, cb);
      acc_a = (row_start ? 1.f : acc_a) * ca;
      carry = new_carry;
      if (HAS_CARRY_OUT && tid == 0 && ((REV ? off : off + CH) % L) == 0) {
        carry_a[row] = acc_a;
        carry_b[row] = carry;
      }
    } else if (HAS_CARRY_OUT && valid && seg_lane_t == tpr - 1) {
      carry_a[row] = pa * a[V - 1];
      carry_b[row] = yv[V - 1];
    }
  }

  if (aborted && tid == 0) {
    // Let copies already in flight land before the CTA's shared memory is
    // released.
    for (int64_t kk = k; kk < issued; ++kk)
      mbar_wait_bounded(&s_bar[kk % S], (uint32_t)((kk / S) & 1));
  }
}

template <typename T>
static int64_t pick_rows_per_tile(int64_t rows, int64_t L, int num_sms) {
  constexpr int CH = kThreads * Elem<T>::kVec;
  const int64_t target = 8 * (int64_t)CH;  // ~32 KiB of each tensor per CTA
  int64_t rpt = target / L;
  const int64_t min_tiles = 4LL * num_sms;
  const int64_t cap = rows / min_tiles;
  if (rpt > cap) rpt = cap;
  if (rpt < 1) rpt = 1;
  return rpt;
}

template <typename T, bool REV, bool HAS_OUT, bool HAS_INIT, bool HAS_CARRY_OUT>
static cudaError_t launch_fwd_t(const FwdArgs& a) {
  const int64_t rpt = pick_rows_per_tile<T>(a.rows, a.seqlen, a.num_sms);
  const int64_t tiles = (a.rows + rpt - 1) / rpt;
  scan_fwd_kernel<T, REV, HAS_OUT, HAS_INIT, HAS_CARRY_OUT>
      <<<(unsigned)tiles, kThreads, 0, a.stream>>>(
          static_cast<const T*>(a.gates), static_cast<const T*>(a.tokens),
          static_cast<T*>(a.out), a.init, a.carry_a, a.carry_b, a.rows, a.seqlen, rpt);
  return cudaGetLastError();
}

template <typename T>
static cudaError_t launch_fwd_dtype(const FwdArgs& a) {
  const bool has_out = a.out != nullptr;
  const bool has_init = a.init != nullptr;
  const bool has_co = a.carry_a != nullptr;
  // Instantiated variants: plain scan (fwd/rev), scan with init (+carry-out),
  // carry-out only (reduce).
  if (has_out && !has_init && !has_co)
    return a.reverse ? launch_fwd_t<T, true, true, false, false>(a)
                     : launch_fwd_t<T, false, true, false, false>(a);
  if (has_out && has_init && !has_co)
    return a.reverse ? launch_fwd_t<T, true, true, true, false>(a)
                     : launch_fwd_t<T, false, true, true, false>(a);
  if (has_out && has_init && has_co)
    return a.reverse ? launch_fwd_t<T, true, true, true, true>(a)
                     : launch_fwd_t<T, false, true, true, true>(a);
  if (has_out && !has_init && has_co)
    return a.reverse ? launch_fwd_t<T, true, true, false, true>(a)
                     : launch_fwd_t<T, false, true, false, true>(a);
  if (!has_out && !has_init && has_co)
    return a.reverse ? launch_fwd_t<T, true, false, false, true>(a)
                     : launch_fwd_t<T, false, false, false, true>(a);
  if (!has_out && has_init && has_co)
    return a.reverse ? launch_fwd_t<T, true, false, true, true>(a)
                     : launch_fwd_t<T, false, false, true, true>(a);
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
