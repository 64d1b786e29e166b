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
// Pipeline, segmentation of short rows and carry handling are the same as in
// scan_fwd.cu.  Optional per-row `addend` (value entering at the row's last
// element, i.e. gates[L] * dtokens[L] of the next sequence shard) and
// `y_prev` (y before the row's first element, from the previous shard) serve
// the sequence-sharded mode; reduce mode (no outputs) emits per row
// gates[0] * dtokens[0], the value the previous shard needs.
#include "common.cuh"
#include "internal.h"

namespace fpscan {

constexpr int kBwdStages = 4;

template <bool HAS_OUT>
constexpr int bwd_smem_bytes() {
  return kBwdStages * 16 * ((kThreads + 1) + kThreads + (HAS_OUT ? kThreads + 1 : 0));
}

template <typename T, bool HAS_OUT, bool HAS_CARRY>
__global__ void __launch_bounds__(kThreads)
    scan_bwd_kernel(const T* __restrict__ gates, const T* __restrict__ y,
                    const T* __restrict__ gout, T* __restrict__ dgates, T* __restrict__ dtok,
                    const float* __restrict__ addend, const float* __restrict__ y_prev,
                    float* __restrict__ carry_b, int64_t rows, int64_t L,
                    int64_t rows_per_tile) {
  constexpr int V = Elem<T>::kVec;
  constexpr int CH = kThreads * V;
  constexpr int S = kBwdStages;
  constexpr int GS = kThreads + 1;  // gates stage: chunk + one vector after
  constexpr int YS = kThreads + 1;  // y stage: one vector before + chunk

  extern __shared__ __align__(128) uint4 dsm[];
  uint4* s_g = dsm;                    // [S][GS]
  uint4* s_go = s_g + S * GS;          // [S][kThreads]
  uint4* s_y = s_go + S * kThreads;    // [S][YS]   (HAS_OUT only)
  __shared__ __align__(8) uint64_t s_bar[S];
  __shared__ float s_wa[2][kWarps], s_wb[2][kWarps];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t row0 = (int64_t)blockIdx.x * rows_per_tile;
  const int64_t nrows = min(rows_per_tile, rows - row0);
  const int64_t base = row0 * L;
  const int64_t n = nrows * L;
  const int64_t nck = (n + CH - 1) / CH;

  const bool multi = L > CH;
  const int tpr = multi ? kThreads : (int)(L / V);
  const int wwidth = tpr < 32 ? tpr : 32;
  const int seg_warps = tpr >> 5;

  if (tid == 0) {
#pragma unroll
    for (int s = 0; s < S; ++s) mbar_init(&s_bar[s], 1);
    fence_mbar_init();
  }
  __syncthreads();

  int64_t issued = 0;
  auto issue = [&](int64_t k) {
    const int64_t mc = nck - 1 - k;  // reverse processing order
    const int64_t off = mc * CH;
    const int64_t cnt = min((int64_t)CH, n - off);
    const uint32_t bytes = (uint32_t)(cnt * (int64_t)sizeof(T));
    const uint32_t g_bytes = bytes + ((off + cnt < n) ? 16u : 0u);
    const int s = (int)(k % S);
    uint32_t y_bytes = 0;
    if (HAS_OUT) y_bytes = bytes + (off > 0 ? 16u : 0u);
    mbar_expect_tx(&s_bar[s], g_bytes + bytes + y_bytes);
    bulk_g2s(s_g + s * GS, gates + base + off, g_bytes, &s_bar[s]);
    bulk_g2s(s_go + s * kThreads, gout + base + off, bytes, &s_bar[s]);
    if (HAS_OUT) {
      if (off > 0)
        bulk_g2s(s_y + s * YS, y + base + off - V, y_bytes, &s_bar[s]);
      else
        bulk_g2s(s_y + s * YS + 1, y + base + off, y_bytes, &s_bar[s]);
    }
  };
  if (tid == 0) {
    for (; issued < min((int64_t)S, nck); ++issued) issue(issued);
  }

  const int vi = kThreads - 1 - tid;
  const int seg_lane_t = tid & (tpr - 1);
  float carry = 0.f;
  int64_t k = 0;
  bool aborted = false;

  for (; k < nck; ++k) {
    const int s = (int)(k % S);
    const uint32_t parity = (uint32_t)((k / S) & 1);
    const int64_t mc = nck - 1 - k;
    const int64_t off = mc * CH;
    const int64_t cnt = min((int64_t)CH, n - off);
    const bool valid = (int64_t)vi * V < cnt;
    const int64_t vstart = off + (int64_t)vi * V;       // tile-relative first element
    const bool vec_row_end = ((vstart + V) % L) == 0;   // vector holds a row's last element
    const bool vec_row_first = (vstart % L) == 0;       // vector holds a row's first element

    const bool ok = mbar_wait_bounded(&s_bar[s], parity);

    Vec16<T> gv, gov;
    float g_next = 1.f;
    float a[V], b[V];
    if (valid) {
      gv.raw = s_g[s * GS + vi];
      gov.raw = s_go[s * kThreads + vi];
      if (!vec_row_end) g_next = Elem<T>::load(reinterpret_cast<const T*>(s_g + s * GS + vi + 1)[0]);
#pragma unroll
      for (int i = 0; i < V; ++i) {
        const int j = V - 1 - i;
        const float g = (j == V - 1) ? g_next : Elem<T>::load(gv.e[j + 1]);
        const float x = Elem<T>::load(gov.e[j]);
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

    // y values needed for dgates, read before the stage is released.
    Vec16<T> yv_own;
    float y_before = 0.f;
    if (HAS_OUT && valid) {
      yv_own.raw = s_y[s * YS + vi + 1];
      if (!vec_row_first)
        y_before = Elem<T>::load(reinterpret_cast<const T*>(s_y + s * YS + vi + 1)[-1]);
    }

    if (__syncthreads_or(!ok)) {
      aborted = true;
      break;
    }
    if (tid == 0 && issued < nck) {
      issue(issued);
      ++issued;
    }

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

    const bool row_start = multi ? (((off + CH) % L) == 0) : true;  // processing order
    const int64_t row = row0 + (multi ? off : vstart) / L;
    float state;
    bool skip_state = false;
    if (row_start) {
      if (HAS_CARRY) {
        carry = addend[row];
        state = fmaf(pa, carry, pb);
      } else {
        carry = 0.f;
        state = pb;
        skip_state = seg_lane_t == 0;
      }
    } else {
      state = fmaf(pa, carry, pb);
    }

    float dt[V];
#pragma unroll
    for (int i = 0; i < V; ++i) dt[i] = skip_state ? b[i] : fmaf(a[i], state, b[i]);

    if (valid) {
      if (HAS_OUT) {
        float yp_first = y_before;
        if (vec_row_first) yp_first = HAS_CARRY ? y_prev[row] : 0.f;
        Vec16<T> o_dt, o_dg;
#pragma unroll
        for (int i = 0; i < V; ++i) {
          const int j = V - 1 - i;
          const float yp = (j == 0) ? yp_first : Elem<T>::load(yv_own.e[j - 1]);
          o_dt.e[j] = Elem<T>::store(dt[i]);
          o_dg.e[j] = Elem<T>::store(dt[i] * yp);
        }
        reinterpret_cast<uint4*>(dtok + base + off)[vi] = o_dt.raw;
        reinterpret_cast<uint4*>(dgates + base + off)[vi] = o_dg.raw;
      } else if (vec_row_first) {
        carry_b[row] = Elem<T>::load(gv.e[0]) * dt[V - 1];
      }
    }

    if (multi) carry = (row_start && !HAS_CARRY) ? cb : fmaf(ca, carry, cb);
  }

  if (aborted && tid == 0) {
    for (int64_t kk = k; kk < issued; ++kk)
      mbar_wait_bounded(&s_bar[kk % S], (uint32_t)((kk / S) & 1));
  }
}

template <typename T>
static int64_t bwd_rows_per_tile(int64_t rows, int64_t L, int num_sms) {
  constexpr int CH = kThreads * Elem<T>::kVec;
  int64_t rpt = (8 * (int64_t)CH) / L;
  const int64_t cap = rows / (4LL * num_sms);
  if (rpt > cap) rpt = cap;
  if (rpt < 1) rpt = 1;
  return rpt;
}

template <typename T, bool HAS_OUT, bool HAS_CARRY>
static cudaError_t launch_bwd_t(const BwdArgs& a) {
  constexpr int smem = bwd_smem_bytes<HAS_OUT>();
  auto kern = scan_bwd_kernel<T, HAS_OUT, HAS_CARRY>;
  // Idempotent and cheap; required because the stage ring exceeds 48 KiB.
  static thread_local int configured_dev = -1;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (configured_dev != dev) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    configured_dev = dev;
  }
  const int64_t rpt = bwd_rows_per_tile<T>(a.rows, a.seqlen, a.num_sms);
  const int64_t tiles = (a.rows + rpt - 1) / rpt;
  kern<<<(unsigned)tiles, kThreads, smem, a.stream>>>(
      static_cast<const T*>(a.gates), static_cast<const T*>(a.y),
      static_cast<const T*>(a.grad_out), static_cast<T*>(a.dgates), static_cast<T*>(a.dtokens),
      a.addend, a.y_prev, a.carry_b, a.rows, a.seqlen, rpt);
  return cudaGetLastError();
}

template <typename T>
static cudaError_t launch_bwd_dtype(const BwdArgs& a) {
  const bool has_out = a.dtokens != nullptr;
  const bool has_carry = a.addend != nullptr;
  if (has_out)
    return has_carry ? launch_bwd_t<T, true, true>(a) : launch_bwd_t<T, true, false>(a);
  return has_carry ? launch_bwd_t<T, false, true>(a) : launch_bwd_t<T, false, false>(a);
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
