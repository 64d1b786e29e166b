// Channel-last scan: forward / reverse scan and fused backward on
// (batch, seqlen, dim) tensors, recurrence along the middle axis, sm_100a.
//
// The reference scans only the last axis; its README (README.md:94-99) has
// channel-last callers transpose with .mT.contiguous() before and after the
// call -- four extra passes over memory.  Here the scan runs on the
// channel-last tensor in place of those passes.
//
// Tile = 32 consecutive 16-byte channel vectors (512 bytes per timestep row:
// 128 fp32 / 256 half channels) x TS timesteps of one batch.  One 3-D TMA
// tensor load per operand stages the tile in shared memory (rows past the
// sequence's ends read as zeros, which also provides y[-1] = 0 and the
// ignored gates[L] of the backward); warp w scans timesteps
// [w*TS/8, (w+1)*TS/8) of all 32 vectors, one lane per vector, reading
// whole 512-byte rows (conflict-free); the warps' per-channel maps are
// combined through shared memory.  Tiles are taken in order from an atomic
// ticket counter, all columns' first segments first, and each tile's
// carry-in comes from a decoupled look-back over the preceding segments of
// its column (per-channel aggregates / inclusive states in the caller's
// workspace, epoch-tagged so it needs no clearing).  DRAM traffic: the
// algorithmic 2 reads + 1 write (forward), 3 + 2 (backward), plus the
// status records (4 / (TS * itemsize) of the data, read back from L2).
//
// Head (zero initial state, gate ignored as at csrc/full_scan/full_scan.cu:96):
// timestep 0 (forward) or L-1 (reverse scan and backward).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cstring>

#include "common.cuh"
#include "internal.h"

namespace fpscan {

namespace {

constexpr int kLanesPerRow = 32;            // 16-byte vectors per tile row
constexpr int kRowBytes = kLanesPerRow * 16;

enum ClMode : int { kClFwd = 0, kClRev = 1, kClBwd = 2 };

struct ClParams {
  CUtensorMap tm_a;  // gates (forward), gates (backward, read one row ahead)
  CUtensorMap tm_b;  // tokens (forward), grad_out (backward)
  CUtensorMap tm_c;  // y (backward, read one row behind)
  void* out;         // y (forward), dtokens (backward)
  void* out2;        // dgates (backward)
  unsigned long long* counter;
  unsigned char* status;
  int64_t L;
  int64_t dv;        // 16-byte vectors per timestep row (dim / V)
  int64_t cb;        // column blocks per batch (ceil(dv / 32))
  int64_t ncol;      // batch * cb
  int64_t segs;      // segments per column (ceil(L / TS))
  uint32_t epoch;
};

// Status record of one tile: flag (epoch << 1 | inclusive), then per channel
// the aggregate map (A, B) and the inclusive state.
template <int V>
struct ClStatus {
  static constexpr int kAgg = 16;
  static constexpr int kIncl = kAgg + kLanesPerRow * V * 8;
  static constexpr int kBytes = kIncl + kLanesPerRow * V * 4;
};

__device__ __forceinline__ void st_release_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Non-multicast 3-D TMA tile load global -> shared, completing on `bar`.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* tm, int x, int y, int z,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
      : "memory");
}

template <typename T>
__device__ __forceinline__ void unpack(const uint4& r, float* f) {
  Vec16<T> v;
  v.raw = r;
#pragma unroll
  for (int c = 0; c < Elem<T>::kVec; ++c) f[c] = Elem<T>::load(v.e[c]);
}

// Warp roles of the channel-last kernel: 8 scan warps, one look-back warp,
// one producer warp.
constexpr int kClScanWarps = kWarps;
constexpr int kClLookbackWarp = kClScanWarps;
constexpr int kClProducerWarp = kClScanWarps + 1;
constexpr int kClThreads = (kClScanWarps + 2) * 32;
constexpr int kClStages = 3;  // TMA ring: tile k+1 scanned, tile k finished, tile k+2 loading

template <typename T, int MODE, int TS>
struct ClCfg {
  static constexpr int kTiles = MODE == kClBwd ? 3 : 2;
  static constexpr int V = Elem<T>::kVec;
  static constexpr int kTileBytes = TS * kRowBytes;
  static constexpr int kStageBytes = kTiles * kTileBytes;               // one tile's operands
  static constexpr int kTotBytes = kClScanWarps * kLanesPerRow * V * 8;  // per-warp maps
  static constexpr int kCarryBytes = kLanesPerRow * V * 4;
  // + 128: the base is rounded up to the 128-byte alignment TMA tensor
  // copies require (dynamic shared memory follows the static variables)
  static constexpr int smem() {
    return kClStages * kStageBytes + 2 * kTotBytes + 2 * kCarryBytes + 128;
  }
};

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}


// Persistent, warp-specialised:
//   producer warp   takes tickets in order and issues each tile's TMA loads
//                   into a 3-stage ring (full / empty mbarriers);
//   scan warps      pass 1 of tile k+1 (per-thread maps -> shared memory),
//                   then, once tile k's carry is known, pass 2 of tile k
//                   (rerun the recurrence, store), then release its stage;
//   look-back warp  composes tile k's aggregate from the scan warps' maps,
//                   publishes it, looks back, publishes the inclusive state
//                   and hands the carry to the scan warps -- while they scan
//                   tile k+1.
// Tickets are taken in order and each CTA finishes its tiles in order, so
// the smallest unfinished ticket always belongs to a CTA that is working on
// it and every look-back ends.  Every wait is bounded (mbarriers only, no
// named barriers); a wait that gives up records a status bit and makes all
// roles of the CTA stop (the others' waits then give up in turn).
template <typename T, int MODE, int TS>
__global__ void __launch_bounds__(kClThreads, 1) scan_cl_kernel(const __grid_constant__ ClParams p) {
  using Cfg = ClCfg<T, MODE, TS>;
  constexpr int V = Elem<T>::kVec;
  constexpr int TW = TS / kClScanWarps;  // timesteps per scan warp
  constexpr bool DESC = MODE != kClFwd;
  constexpr bool BWD = MODE == kClBwd;
  constexpr int S = kClStages;
  using St = ClStatus<V>;
  static_assert(TS % kClScanWarps == 0, "TS must be a multiple of the scan warp count");

  extern __shared__ __align__(128) unsigned char csm_raw[];
  unsigned char* csm = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(csm_raw) + 127) & ~uintptr_t(127));
  float2* s_tot_base = reinterpret_cast<float2*>(csm + S * Cfg::kStageBytes);  // [2][8][32][V]
  float* s_carry_base =
      reinterpret_cast<float*>(csm + S * Cfg::kStageBytes + 2 * Cfg::kTotBytes);  // [2][32][V]
  // full/empty: TMA ring; totb: scan warps' maps of a tile written; carryb:
  // its carry written; consumed: maps and carry read (buffer h reusable)
  __shared__ __align__(8) uint64_t s_full[S], s_empty[S], s_totb[2], s_carryb[2], s_consumed[2];
  __shared__ long long s_tk[S];
  __shared__ int s_hf[2][kClScanWarps];
  __shared__ volatile int s_abort;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t ntiles = p.ncol * p.segs;
  const int64_t L = p.L;
  const int64_t head_t = DESC ? L - 1 : 0;
  // TMA tensor copies need a 128-byte aligned destination: checked, never
  // assumed (a failed check stops the CTA like a copy that never lands)
  const bool aligned = (smem_addr(csm) & 127u) == 0;

  auto coords = [&](int64_t ticket, int64_t& seg_p, int64_t& b, int64_t& cblk, int64_t& s0) {
    seg_p = ticket / p.ncol;
    const int64_t col = ticket - seg_p * p.ncol;
    b = col / p.cb;
    cblk = col - b * p.cb;
    s0 = (DESC ? p.segs - 1 - seg_p : seg_p) * TS;
  };

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&s_empty[s], kClScanWarps * 32);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_totb[i], kClScanWarps * 32);
      mbar_init(&s_carryb[i], 32);
      mbar_init(&s_consumed[i], kClScanWarps * 32);
    }
    fence_mbar_init();
    s_abort = aligned ? 0 : 1;
    if (!aligned) atomicOr(&g_status, kStatusMisaligned);
  }
  __syncthreads();
  if (s_abort) return;

  // ================================================================ producer
  if (warp == kClProducerWarp) {
    if (lane != 0) return;
    for (int64_t k = 0;; ++k) {
      const int s = (int)(k % S);
      if (k >= S && !mbar_wait_bounded(&s_empty[s], (uint32_t)((k / S - 1) & 1))) {
        s_abort = 1;
        return;
      }
      if (s_abort) return;
      const long long t = (long long)atomicAdd(p.counter, 1ull);
      s_tk[s] = t;
      if (t >= ntiles) {
        mbar_expect_tx(&s_full[s], 0u);  // wakes the consumers with the end marker
        return;
      }
      int64_t seg_p, b, cblk, s0;
      coords(t, seg_p, b, cblk, s0);
      unsigned char* dst = csm + s * Cfg::kStageBytes;
      const int x = (int)(cblk * kLanesPerRow * V);
      mbar_expect_tx(&s_full[s], (uint32_t)Cfg::kStageBytes);
      if (BWD) {
        tma_load_3d(dst, &p.tm_a, x, (int)(s0 + 1), (int)b, &s_full[s]);
        tma_load_3d(dst + Cfg::kTileBytes, &p.tm_b, x, (int)s0, (int)b, &s_full[s]);
        tma_load_3d(dst + 2 * Cfg::kTileBytes, &p.tm_c, x, (int)(s0 - 1), (int)b, &s_full[s]);
      } else {
        tma_load_3d(dst, &p.tm_a, x, (int)s0, (int)b, &s_full[s]);
        tma_load_3d(dst + Cfg::kTileBytes, &p.tm_b, x, (int)s0, (int)b, &s_full[s]);
      }
    }
  }

  // ================================================================ look-back
  if (warp == kClLookbackWarp) {
    for (int64_t k = 0;; ++k) {
      const int s = (int)(k % S), h = (int)(k & 1);
      // decisions are warp-uniform: the warp later uses __syncwarp/__all_sync
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(&s_full[s], (uint32_t)((k / S) & 1))) ||
          __any_sync(0xffffffffu, s_abort != 0)) {
        s_abort = 1;
        return;
      }
      const int64_t ticket = s_tk[s];
      if (ticket >= ntiles) return;
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(&s_totb[h], (uint32_t)((k >> 1) & 1))) ||
          __any_sync(0xffffffffu, s_abort != 0)) {
        s_abort = 1;
        return;
      }
      const int64_t seg_p = ticket / p.ncol;
      // tile aggregate per channel from the scan warps' maps (processing order)
      const float2* tot = s_tot_base + (size_t)h * kClScanWarps * kLanesPerRow * V;
      int q0 = 0;
      bool gf = false;
      for (int q = 0; q < kClScanWarps; ++q)
        if (s_hf[h][q]) {
          q0 = q;
          gf = true;
        }
      float GA[V], GB[V];
      for (int q = q0; q < kClScanWarps; ++q) {
        const float2* t = tot + (q * kLanesPerRow + lane) * V;
#pragma unroll
        for (int c = 0; c < V; ++c) {
          const float2 m = t[c];
          if (q == q0) {
            GA[c] = m.x;
            GB[c] = m.y;
          } else {
            GB[c] = fmaf(GB[c], m.x, m.y);
            GA[c] *= m.x;
          }
        }
      }

      unsigned char* rec = p.status + ticket * (int64_t)St::kBytes;
      uint32_t* flag = reinterpret_cast<uint32_t*>(rec);
      float* incl = reinterpret_cast<float*>(rec + St::kIncl) + lane * V;
      const uint32_t agg_flag = p.epoch << 1, incl_flag = (p.epoch << 1) | 1u;
      float carry[V];
#pragma unroll
      for (int c = 0; c < V; ++c) carry[c] = 0.f;

      auto publish = [&](const float* src_a, const float* src_b, bool inclusive) {
        if (inclusive) {
#pragma unroll
          for (int c = 0; c < V; c += 4)
            *reinterpret_cast<float4*>(incl + c) =
                make_float4(src_b[c], src_b[c + 1], src_b[c + 2], src_b[c + 3]);
        } else {
          float* agg = reinterpret_cast<float*>(rec + St::kAgg) + lane * V * 2;
#pragma unroll
          for (int c = 0; c < V; c += 2)
            *reinterpret_cast<float4*>(agg + 2 * c) =
                make_float4(src_a[c], src_b[c], src_a[c + 1], src_b[c + 1]);
        }
        __threadfence();
        __syncwarp();
        if (lane == 0) st_release_u32(flag, inclusive ? incl_flag : agg_flag);
      };

      if (gf || seg_p == 0) {
        // the tile holds the head: its inclusive state needs no carry
        publish(GA, GB, true);
      } else {
        const unsigned char* prev = p.status + (ticket - p.ncol) * (int64_t)St::kBytes;
        const uint32_t f0 = ld_acquire_u32(reinterpret_cast<const uint32_t*>(prev));
        const bool direct = __all_sync(0xffffffffu, f0 == incl_flag);
        if (!direct) publish(GA, GB, false);
        float acc_a[V], acc_b[V];  // composition of the tiles passed over
        bool acc_have = false;
        const uint64_t t_start = global_ns();
        for (int64_t j = ticket - p.ncol; j >= 0; j -= p.ncol) {
          const unsigned char* r = p.status + j * (int64_t)St::kBytes;
          const uint32_t* fj = reinterpret_cast<const uint32_t*>(r);
          uint32_t f = ld_acquire_u32(fj);
          uint32_t spins = 0;
          bool timed_out = false;
          while ((f >> 1) != p.epoch) {
            if ((++spins & 63u) == 0 && global_ns() - t_start > kWaitLimitNs) {
              timed_out = true;
              break;
            }
            f = ld_acquire_u32(fj);
          }
          if (timed_out) {
            atomicOr(&g_status, kStatusLookbackTimeout);
            break;  // carry stays 0
          }
          if (f & 1u) {
            const float* ji = reinterpret_cast<const float*>(r + St::kIncl) + lane * V;
#pragma unroll
            for (int c = 0; c < V; c += 4) {
              const float4 v = __ldcg(reinterpret_cast<const float4*>(ji + c));
              const float vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
              for (int u = 0; u < 4; ++u)
                carry[c + u] = acc_have ? fmaf(acc_a[c + u], vv[u], acc_b[c + u]) : vv[u];
            }
            break;
          }
          const float* ja = reinterpret_cast<const float*>(r + St::kAgg) + lane * V * 2;
#pragma unroll
          for (int c = 0; c < V; c += 2) {
            const float4 v = __ldcg(reinterpret_cast<const float4*>(ja + 2 * c));
            if (!acc_have) {
              acc_a[c] = v.x;
              acc_b[c] = v.y;
              acc_a[c + 1] = v.z;
              acc_b[c + 1] = v.w;
            } else {
              acc_b[c] = fmaf(v.y, acc_a[c], acc_b[c]);
              acc_a[c] *= v.x;
              acc_b[c + 1] = fmaf(v.w, acc_a[c + 1], acc_b[c + 1]);
              acc_a[c + 1] *= v.z;
            }
          }
          acc_have = true;
        }
        float st_incl[V];
#pragma unroll
        for (int c = 0; c < V; ++c) st_incl[c] = fmaf(GA[c], carry[c], GB[c]);
        publish(GA, st_incl, true);
      }
      float* sc = s_carry_base + (size_t)h * kLanesPerRow * V + lane * V;
#pragma unroll
      for (int c = 0; c < V; ++c) sc[c] = carry[c];
      mbar_arrive(&s_carryb[h]);
    }
  }

  // ================================================================ scan warps
  const int pw = warp;  // scan warp index = its place in processing order
  T* out = static_cast<T*>(p.out);
  T* out2 = static_cast<T*>(p.out2);
  const int64_t row_elems = p.dv * V;

  // pass 1 of tile k (stage k % S): per-thread maps to s_tot[k & 1]
  auto pass1 = [&](int64_t k, int64_t ticket) -> bool {
    const int s = (int)(k % S), h = (int)(k & 1);
    // buffer h last held tile k-2: wait until every scan thread has read it
    if (k >= 2 && !mbar_wait_bounded(&s_consumed[h], (uint32_t)(((k - 2) >> 1) & 1))) return false;
    int64_t seg_p, b, cblk, s0;
    coords(ticket, seg_p, b, cblk, s0);
    const uint4* s_a = reinterpret_cast<const uint4*>(csm + s * Cfg::kStageBytes);
    const uint4* s_b = reinterpret_cast<const uint4*>(csm + s * Cfg::kStageBytes + Cfg::kTileBytes);
    float A[V], B[V];
    bool hf = false;
#pragma unroll
    for (int i = 0; i < TW; ++i) {
      const int lr = DESC ? TS - 1 - (pw * TW + i) : pw * TW + i;
      float g[V], x[V];
      unpack<T>(s_a[lr * kLanesPerRow + lane], g);
      unpack<T>(s_b[lr * kLanesPerRow + lane], x);
      const bool head = s0 + lr == head_t;
#pragma unroll
      for (int c = 0; c < V; ++c) {
        if (i == 0) {
          A[c] = g[c];
          B[c] = x[c];
        } else {
          B[c] = fmaf(B[c], g[c], x[c]);
          A[c] *= g[c];
        }
        if (head) {
          A[c] = 1.f;
          B[c] = x[c];
        }
      }
      hf |= head;
    }
    float2* tot = s_tot_base + (size_t)h * kClScanWarps * kLanesPerRow * V;
#pragma unroll
    for (int c = 0; c < V; ++c) tot[(pw * kLanesPerRow + lane) * V + c] = make_float2(A[c], B[c]);
    if (lane == 0) s_hf[h][pw] = hf ? 1 : 0;
    mbar_arrive(&s_totb[h]);  // release: orders this thread's writes above
    return true;
  };

  // pass 2 of tile k: prefix over earlier warps, carry, rerun, store
  auto pass2 = [&](int64_t k, int64_t ticket) {
    const int s = (int)(k % S), h = (int)(k & 1);
    int64_t seg_p, b, cblk, s0;
    coords(ticket, seg_p, b, cblk, s0);
    const float2* tot = s_tot_base + (size_t)h * kClScanWarps * kLanesPerRow * V;
    float EA[V], EB[V];
    bool have = false, ef = false;
    int q0 = 0;
    for (int q = 0; q < pw; ++q)
      if (s_hf[h][q]) {
        q0 = q;
        ef = true;
      }
    for (int q = q0; q < pw; ++q) {
      const float2* t = tot + (q * kLanesPerRow + lane) * V;
#pragma unroll
      for (int c = 0; c < V; ++c) {
        const float2 m = t[c];
        if (!have) {
          EA[c] = m.x;
          EB[c] = m.y;
        } else {
          EB[c] = fmaf(EB[c], m.x, m.y);
          EA[c] *= m.x;
        }
      }
      have = true;
    }
    float st[V];
    const float* sc = s_carry_base + (size_t)h * kLanesPerRow * V + lane * V;
#pragma unroll
    for (int c = 0; c < V; ++c) {
      const float cin = sc[c];
      st[c] = ef ? EB[c] : (have ? fmaf(EA[c], cin, EB[c]) : cin);
    }
    // this thread has read s_tot[h], s_hf[h] and s_carry[h]
    mbar_arrive(&s_consumed[h]);
    const uint4* s_a = reinterpret_cast<const uint4*>(csm + s * Cfg::kStageBytes);
    const uint4* s_b = reinterpret_cast<const uint4*>(csm + s * Cfg::kStageBytes + Cfg::kTileBytes);
    const uint4* s_c =
        reinterpret_cast<const uint4*>(csm + s * Cfg::kStageBytes + 2 * Cfg::kTileBytes);
    const int64_t cv = cblk * kLanesPerRow + lane;
    const bool lane_ok = cv < p.dv;
    const int64_t base = (b * L) * row_elems + cv * V;
#pragma unroll
    for (int i = 0; i < TW; ++i) {
      const int lr = DESC ? TS - 1 - (pw * TW + i) : pw * TW + i;
      const int64_t t = s0 + lr;
      float g[V], x[V];
      unpack<T>(s_a[lr * kLanesPerRow + lane], g);
      unpack<T>(s_b[lr * kLanesPerRow + lane], x);
      const bool head = t == head_t;
#pragma unroll
      for (int c = 0; c < V; ++c) st[c] = head ? x[c] : fmaf(g[c], st[c], x[c]);
      if (t < L && lane_ok) {
        *reinterpret_cast<uint4*>(out + base + t * row_elems) = pack_vec<T>(st);
        if (BWD) {
          float yp[V], dg[V];
          unpack<T>(s_c[lr * kLanesPerRow + lane], yp);
#pragma unroll
          for (int c = 0; c < V; ++c) dg[c] = st[c] * yp[c];
          *reinterpret_cast<uint4*>(out2 + base + t * row_elems) = pack_vec<T>(dg);
        }
      }
    }
    mbar_arrive(&s_empty[s]);
  };

  if (!mbar_wait_bounded(&s_full[0], 0) || s_abort) {
    s_abort = 1;
    return;
  }
  int64_t ticket = s_tk[0];
  if (ticket >= ntiles) return;
  pass1(0, ticket);  // k = 0 waits for nothing
  for (int64_t k = 0;; ++k) {
    const int sn = (int)((k + 1) % S);
    if (!mbar_wait_bounded(&s_full[sn], (uint32_t)(((k + 1) / S) & 1)) || s_abort) {
      s_abort = 1;
      return;
    }
    const int64_t next = s_tk[sn];
    if (next < ntiles && !pass1(k + 1, next)) {
      s_abort = 1;
      return;
    }
    if (!mbar_wait_bounded(&s_carryb[k & 1], (uint32_t)((k >> 1) & 1)) || s_abort) {
      s_abort = 1;
      return;
    }
    pass2(k, ticket);
    if (next >= ntiles) return;
    ticket = next;
  }
}

// ------------------------------------------------------------------ streaming
// Column-streaming channel-last kernel, used when there are enough columns
// for every CTA slot: one CTA per column of kStreamVecs 16-byte channel
// vectors (128-byte rows), streamed chunk by chunk through a kStages-deep
// TMA ring (one elected thread refills a stage right after the chunk's
// single __syncthreads), with the state carried across
// chunks in shared memory -- no look-back and no workspace.  Pass 2 rereads
// the chunk from shared memory, so a stage is refilled one chunk later than
// in scan_fwd.cu (S - 1 chunks in flight ahead of the one scanned).  A chunk is
// 32 thread groups x TW timesteps; thread (warp w, lane) owns channel
// vector lane % 8 and timesteps [(4w + lane/8) * TW, +TW) of the chunk.
// Reading whole 128-byte rows per 8 lanes is bank-conflict free.
constexpr int kStreamVecs = 8;
constexpr int kStreamRowBytes = kStreamVecs * 16;

template <typename T, int MODE, int TW, int S, int NTH>
struct StreamCfg {
  static constexpr int NW = NTH / 32;          // warps
  static constexpr int NG = NTH / kStreamVecs;  // thread groups
  static constexpr int kTiles = MODE == kClBwd ? 3 : 2;
  static constexpr int R = NG * TW;  // timesteps per chunk
  static constexpr int kTileBytes = R * kStreamRowBytes;
  static constexpr int kStageBytes = kTiles * kTileBytes;
  static constexpr int smem() { return S * kStageBytes + 128; }  // + TMA alignment slack
};

struct StreamParams {
  CUtensorMap tm_a, tm_b, tm_c;  // as ClParams
  void* out;
  void* out2;
  int64_t L;
  int64_t dv;    // 16-byte vectors per timestep row
  int64_t cb;    // column blocks per batch (ceil(dv / 8))
};

template <typename T, int MODE, int TW, int S, int NTH>
__global__ void __launch_bounds__(NTH, 1)
    scan_cl_stream_kernel(const __grid_constant__ StreamParams p) {
  using Cfg = StreamCfg<T, MODE, TW, S, NTH>;
  constexpr int NW = Cfg::NW;
  constexpr int V = Elem<T>::kVec;
  constexpr int R = Cfg::R;
  constexpr bool DESC = MODE != kClFwd;
  constexpr bool BWD = MODE == kClBwd;

  extern __shared__ __align__(128) unsigned char csm_raw[];
  unsigned char* csm = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(csm_raw) + 127) & ~uintptr_t(127));
  __shared__ __align__(8) uint64_t s_bar[S];
  // warp maps per channel and vector (vectors innermost: conflict-free), by chunk parity
  __shared__ float2 s_wt[2][NW][V][kStreamVecs];
  __shared__ float s_carry[2][kStreamVecs][V];          // state after a chunk, by chunk parity

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int vec = lane & (kStreamVecs - 1), grp = lane >> 3;
  const int tg = warp * (32 / kStreamVecs) + grp;  // thread group, processing order
  const int64_t col = blockIdx.x;
  const int64_t b = col / p.cb, cblk = col - b * p.cb;
  const int64_t L = p.L;
  const int64_t head_t = DESC ? L - 1 : 0;
  const int64_t nck = (L + R - 1) / R;
  const int64_t cv = cblk * kStreamVecs + vec;
  const bool lane_ok = cv < p.dv;
  const bool aligned = (smem_addr(csm) & 127u) == 0;  // TMA destination rule, checked

  if (tid == 0) {
#pragma unroll
    for (int s = 0; s < S; ++s) mbar_init(&s_bar[s], 1);
    fence_mbar_init();
    if (!aligned) atomicOr(&g_status, kStatusMisaligned);
  }
  __syncthreads();
  if (!aligned) return;

  const int x = (int)(cblk * kStreamVecs * V);
  int64_t issued = 0;
  auto issue = [&](int64_t k) {
    const int64_t m = DESC ? nck - 1 - k : k;
    const int s = (int)(k % S);
    unsigned char* dst = csm + s * Cfg::kStageBytes;
    const int r0 = (int)(m * R);
    mbar_expect_tx(&s_bar[s], (uint32_t)Cfg::kStageBytes);
    if (BWD) {
      tma_load_3d(dst, &p.tm_a, x, r0 + 1, (int)b, &s_bar[s]);
      tma_load_3d(dst + Cfg::kTileBytes, &p.tm_b, x, r0, (int)b, &s_bar[s]);
      tma_load_3d(dst + 2 * Cfg::kTileBytes, &p.tm_c, x, r0 - 1, (int)b, &s_bar[s]);
    } else {
      tma_load_3d(dst, &p.tm_a, x, r0, (int)b, &s_bar[s]);
      tma_load_3d(dst + Cfg::kTileBytes, &p.tm_b, x, r0, (int)b, &s_bar[s]);
    }
  };
  if (tid == 0)
    for (; issued < min((int64_t)S, nck); ++issued) issue(issued);

  T* out = static_cast<T*>(p.out);
  T* out2 = static_cast<T*>(p.out2);
  const int64_t row_elems = p.dv * V;
  const int64_t base = (b * L) * row_elems + cv * V;

  int64_t k = 0;
  int s = 0;
  uint32_t phase = 0;
  bool aborted = false;
  for (; k < nck; ++k) {
    const int64_t m = DESC ? nck - 1 - k : k;
    const int64_t r0 = m * R;
    const bool ok = mbar_wait_bounded(&s_bar[s], phase);
    const uint4* s_a = reinterpret_cast<const uint4*>(csm + s * Cfg::kStageBytes);
    const uint4* s_b = reinterpret_cast<const uint4*>(csm + s * Cfg::kStageBytes + Cfg::kTileBytes);
    const uint4* s_c =
        reinterpret_cast<const uint4*>(csm + s * Cfg::kStageBytes + 2 * Cfg::kTileBytes);

    // pass 1: the thread's map over its TW timesteps
    float A[V], B[V];
#pragma unroll
    for (int i = 0; i < TW; ++i) {
      const int lr = DESC ? R - 1 - (tg * TW + i) : tg * TW + i;
      float g[V], xx[V];
      unpack<T>(s_a[lr * kStreamVecs + vec], g);
      unpack<T>(s_b[lr * kStreamVecs + vec], xx);
      const bool head = r0 + lr == head_t;
#pragma unroll
      for (int c = 0; c < V; ++c) {
        if (i == 0) {
          A[c] = g[c];
          B[c] = xx[c];
        } else {
          B[c] = fmaf(B[c], g[c], xx[c]);
          A[c] *= g[c];
        }
        if (head) {  // gate ignored; the state entering the head is 0 (see below)
          A[c] = 1.f;
          B[c] = xx[c];
        }
      }
    }
    // warp: inclusive scan over the 4 groups of each vector (lanes 8 apart)
#pragma unroll
    for (int d = 1; d < 32 / kStreamVecs; d <<= 1) {
#pragma unroll
      for (int c = 0; c < V; ++c) {
        const float pa = __shfl_up_sync(0xffffffffu, A[c], d * kStreamVecs);
        const float pb = __shfl_up_sync(0xffffffffu, B[c], d * kStreamVecs);
        if (grp >= d) {
          B[c] = fmaf(pb, A[c], B[c]);
          A[c] = pa * A[c];
        }
      }
    }
    float EA[V], EB[V];  // exclusive within the warp
#pragma unroll
    for (int c = 0; c < V; ++c) {
      EA[c] = __shfl_up_sync(0xffffffffu, A[c], kStreamVecs);
      EB[c] = __shfl_up_sync(0xffffffffu, B[c], kStreamVecs);
    }
    const int buf = (int)(k & 1);
    if (grp == 32 / kStreamVecs - 1)
#pragma unroll
      for (int c = 0; c < V; ++c) s_wt[buf][warp][c][vec] = make_float2(A[c], B[c]);

    if (__syncthreads_or(!ok)) {
      aborted = true;
      break;
    }
    // Pass 2 below still reads stage s, but every thread has finished the
    // previous chunk: refill that chunk's stage (issued == k - 1 + S).
    if (tid == 0 && k >= 1 && issued < nck) {
      issue(issued);
      ++issued;
    }

    // state entering the thread's first timestep: carry, then the earlier
    // warps, then the earlier groups of this warp.  Compositions start from
    // real operands.  Before the head every operand is a zero-filled row
    // (rows outside [0, L) read as zeros) and the carry is 0, so the state
    // entering the head is exactly 0.
    // In the first chunk the entering state is exactly 0: maps are applied
    // as their B alone (never A * 0, which an overflowed A would make NaN).
    float st[V];
    bool zero = k == 0;
#pragma unroll
    for (int c = 0; c < V; ++c) st[c] = zero ? 0.f : s_carry[buf ^ 1][vec][c];
    for (int q = 0; q < warp; ++q) {
#pragma unroll
      for (int c = 0; c < V; ++c) {
        const float2 mq = s_wt[buf][q][c][vec];
        st[c] = zero ? mq.y : fmaf(mq.x, st[c], mq.y);
      }
      zero = false;
    }
    if (grp > 0)
#pragma unroll
      for (int c = 0; c < V; ++c) st[c] = zero ? EB[c] : fmaf(EA[c], st[c], EB[c]);

    // pass 2: rerun the recurrence from the entering state, store
#pragma unroll
    for (int i = 0; i < TW; ++i) {
      const int lr = DESC ? R - 1 - (tg * TW + i) : tg * TW + i;
      const int64_t t = r0 + lr;
      float g[V], xx[V];
      unpack<T>(s_a[lr * kStreamVecs + vec], g);
      unpack<T>(s_b[lr * kStreamVecs + vec], xx);
      const bool head = t == head_t;
#pragma unroll
      for (int c = 0; c < V; ++c) st[c] = head ? xx[c] : fmaf(g[c], st[c], xx[c]);
      if (t >= 0 && t < L && lane_ok) {
        *reinterpret_cast<uint4*>(out + base + t * row_elems) = pack_vec<T>(st);
        if (BWD) {
          float yp[V], dg[V];
          unpack<T>(s_c[lr * kStreamVecs + vec], yp);
#pragma unroll
          for (int c = 0; c < V; ++c) dg[c] = st[c] * yp[c];
          *reinterpret_cast<uint4*>(out2 + base + t * row_elems) = pack_vec<T>(dg);
        }
      }
    }
    // the chunk's last timestep (processing order) carries into the next
    if (tg == Cfg::NG - 1)
#pragma unroll
      for (int c = 0; c < V; ++c) s_carry[buf][vec][c] = st[c];

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

// ------------------------------------------------------------------ host side
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      f = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  }();
  return fn;
}

// 3-D map over (dim, seqlen, batch) with a (row_bytes, ts, 1) box.
cudaError_t make_map(CUtensorMap* m, const void* ptr, int dtype, int64_t batch, int64_t L,
                     int64_t dim, int ts, int row_bytes = kRowBytes) {
  auto fn = encode_fn();
  if (!fn) return cudaErrorNotSupported;
  const int es = dtype_size(dtype);
  const CUtensorMapDataType dt = dtype == kF32   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : dtype == kF16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const cuuint64_t dims[3] = {(cuuint64_t)dim, (cuuint64_t)L, (cuuint64_t)batch};
  const cuuint64_t strides[2] = {(cuuint64_t)(dim * es), (cuuint64_t)(L * dim * es)};
  const cuuint32_t box[3] = {(cuuint32_t)(row_bytes / es), (cuuint32_t)ts, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = fn(m, dt, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

uint32_t next_cl_epoch() {
  static std::atomic<uint32_t> ctr{0};
  uint32_t e;
  do {
    e = (ctr.fetch_add(1, std::memory_order_relaxed) + 1) & 0x7fffffffu;
  } while (e == 0);
  return e;
}

// Timesteps per tile.  FPSCAN_B200_CL_TS_FWD / FPSCAN_B200_CL_TS_BWD (16,
// 32 or 64) override the defaults (a tuning knob read once per process).
int cl_tile_steps(bool backward) {
  static const int env_f = [] {
    const char* v = getenv("FPSCAN_B200_CL_TS_FWD");
    return v ? atoi(v) : 0;
  }();
  static const int env_b = [] {
    const char* v = getenv("FPSCAN_B200_CL_TS_BWD");
    return v ? atoi(v) : 0;
  }();
  const int e = backward ? env_b : env_f;
  if (e == 16 || e == 32 || e == 64) return e;
  return 32;
}

template <typename T, int MODE, int TS>
cudaError_t launch_cl_t(const ClArgs& a) {
  constexpr int V = Elem<T>::kVec;
  constexpr int smem = ClCfg<T, MODE, TS>::smem();
  auto kern = scan_cl_kernel<T, MODE, TS>;
  static int occ_cache[64] = {0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  int occ = (dev >= 0 && dev < 64) ? occ_cache[dev] : 0;
  if (occ == 0) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kClThreads, smem) != cudaSuccess ||
        occ < 1)
      occ = 1;
    if (dev >= 0 && dev < 64) occ_cache[dev] = occ;
  }
  int sms = 0;
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  ClParams p;
  memset(&p, 0, sizeof(p));
  const int64_t dv = a.dim / V;
  p.L = a.seqlen;
  p.dv = dv;
  p.cb = (dv + kLanesPerRow - 1) / kLanesPerRow;
  p.ncol = a.batch * p.cb;
  p.segs = (a.seqlen + TS - 1) / TS;
  const int64_t tiles = p.ncol * p.segs;
  if ((int64_t)a.workspace_bytes < cl_workspace_bytes(a.batch, a.seqlen, a.dim, a.dtype, MODE == kClBwd))
    return cudaErrorInvalidValue;
  if (MODE == kClBwd) {
    e = make_map(&p.tm_a, a.gates, a.dtype, a.batch, a.seqlen, a.dim, TS);
    if (e == cudaSuccess) e = make_map(&p.tm_b, a.grad_out, a.dtype, a.batch, a.seqlen, a.dim, TS);
    if (e == cudaSuccess) e = make_map(&p.tm_c, a.y, a.dtype, a.batch, a.seqlen, a.dim, TS);
    p.out = a.dtokens;
    p.out2 = a.dgates;
  } else {
    e = make_map(&p.tm_a, a.gates, a.dtype, a.batch, a.seqlen, a.dim, TS);
    if (e == cudaSuccess) e = make_map(&p.tm_b, a.tokens, a.dtype, a.batch, a.seqlen, a.dim, TS);
    p.out = a.out;
  }
  if (e != cudaSuccess) return e;
  e = cudaMemsetAsync(a.workspace, 0, sizeof(unsigned long long), a.stream);
  if (e != cudaSuccess) return e;
  p.counter = static_cast<unsigned long long*>(a.workspace);
  p.status = static_cast<unsigned char*>(a.workspace) + 256;
  p.epoch = next_cl_epoch();
  const int64_t grid = std::min<int64_t>(tiles, (int64_t)sms * occ);
  kern<<<(unsigned)grid, kClThreads, smem, a.stream>>>(p);
  return cudaGetLastError();
}

template <typename T, int MODE>
cudaError_t launch_cl_mode(const ClArgs& a) {
  switch (cl_tile_steps(MODE == kClBwd)) {
    case 16:
      return launch_cl_t<T, MODE, 16>(a);
    case 64:
      return launch_cl_t<T, MODE, 64>(a);
    default:
      return launch_cl_t<T, MODE, 32>(a);
  }
}

template <typename T, int MODE, int TW, int S, int NTH = kThreads>
cudaError_t launch_stream_t(const ClArgs& a) {
  using Cfg = StreamCfg<T, MODE, TW, S, NTH>;
  constexpr int V = Elem<T>::kVec;
  constexpr int smem = Cfg::smem();
  auto kern = scan_cl_stream_kernel<T, MODE, TW, S, NTH>;
  static int configured[64] = {0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) configured[dev] = 1;
  }
  StreamParams p;
  memset(&p, 0, sizeof(p));
  p.L = a.seqlen;
  p.dv = a.dim / V;
  p.cb = (p.dv + kStreamVecs - 1) / kStreamVecs;
  const int64_t R = Cfg::R;
  if (MODE == kClBwd) {
    e = make_map(&p.tm_a, a.gates, a.dtype, a.batch, a.seqlen, a.dim, R, kStreamRowBytes);
    if (e == cudaSuccess)
      e = make_map(&p.tm_b, a.grad_out, a.dtype, a.batch, a.seqlen, a.dim, R, kStreamRowBytes);
    if (e == cudaSuccess) e = make_map(&p.tm_c, a.y, a.dtype, a.batch, a.seqlen, a.dim, R, kStreamRowBytes);
    p.out = a.dtokens;
    p.out2 = a.dgates;
  } else {
    e = make_map(&p.tm_a, a.gates, a.dtype, a.batch, a.seqlen, a.dim, R, kStreamRowBytes);
    if (e == cudaSuccess)
      e = make_map(&p.tm_b, a.tokens, a.dtype, a.batch, a.seqlen, a.dim, R, kStreamRowBytes);
    p.out = a.out;
  }
  if (e != cudaSuccess) return e;
  const int64_t cols = a.batch * p.cb;
  kern<<<(unsigned)cols, NTH, smem, a.stream>>>(p);
  return cudaGetLastError();
}

// Streaming-kernel shape: TW timesteps per thread group, S ring stages and
// threads per CTA.  Defaults: forward 8x3 (192 KiB of stages), backward 8x2
// (its three operands leave room for two), 256 threads.
// FPSCAN_B200_CL_STREAM=4x4 / 4x3 / 8x2 / 8x3 / w4x3 / w4x2 overrides
// ("w": 512 threads; 8x3 and w4x3 apply to the forward only).
template <typename T, int MODE>
cudaError_t launch_stream_mode(const ClArgs& a) {
  static const int cfg = [] {
    const char* v = getenv("FPSCAN_B200_CL_STREAM");
    if (!v) return 0;
    if (!strcmp(v, "4x4")) return 1;
    if (!strcmp(v, "8x3")) return 2;
    if (!strcmp(v, "4x3")) return 3;
    if (!strcmp(v, "8x2")) return 4;
    if (!strcmp(v, "w4x3")) return 5;
    if (!strcmp(v, "w4x2")) return 6;
    return 0;
  }();
  constexpr bool kBwd = MODE == kClBwd;
  switch (cfg) {
    case 1:
      return launch_stream_t<T, MODE, 4, 4>(a);
    case 3:
      return launch_stream_t<T, MODE, 4, 3>(a);
    case 4:
      return launch_stream_t<T, MODE, 8, 2>(a);
    case 5:
      if constexpr (!kBwd) return launch_stream_t<T, MODE, 4, 3, 512>(a);
      [[fallthrough]];
    case 6:
      return launch_stream_t<T, MODE, 4, 2, 512>(a);
    default:
      if constexpr (kBwd) return launch_stream_t<T, MODE, 8, 2>(a);
      else return launch_stream_t<T, MODE, 8, 3>(a);
  }
}

template <typename T>
cudaError_t launch_cl_dtype(const ClArgs& a) {
  if (cl_use_stream(a.batch, a.dim, a.dtype)) {
    if (a.backward) return launch_stream_mode<T, kClBwd>(a);
    return a.reverse ? launch_stream_mode<T, kClRev>(a) : launch_stream_mode<T, kClFwd>(a);
  }
  if (a.backward) return launch_cl_mode<T, kClBwd>(a);
  return a.reverse ? launch_cl_mode<T, kClRev>(a) : launch_cl_mode<T, kClFwd>(a);
}

}  // namespace

// The streaming kernel needs one CTA per 8-vector column and no workspace;
// it is used when the columns fill the GPU (>= kStreamMinCols), the
// look-back kernel otherwise.  FPSCAN_B200_CL_PATH=stream / lookback forces
// one (tests and measurements).
constexpr int64_t kStreamMinCols = 128;
bool cl_use_stream(int64_t batch, int64_t dim, int dtype) {
  static const int force = [] {
    const char* v = getenv("FPSCAN_B200_CL_PATH");
    if (v && !strcmp(v, "stream")) return 1;
    if (v && !strcmp(v, "lookback")) return 2;
    return 0;
  }();
  if (force) return force == 1;
  const int64_t dv = dim / (16 / dtype_size(dtype));
  return batch * ((dv + kStreamVecs - 1) / kStreamVecs) >= kStreamMinCols;
}

int64_t cl_workspace_bytes(int64_t batch, int64_t seqlen, int64_t dim, int dtype, bool backward) {
  if (cl_use_stream(batch, dim, dtype)) return 256;
  const int es = dtype_size(dtype);
  const int V = 16 / es;
  const int ts = cl_tile_steps(backward);
  const int64_t dv = dim / V;
  const int64_t tiles = batch * ((dv + kLanesPerRow - 1) / kLanesPerRow) * ((seqlen + ts - 1) / ts);
  const int64_t rec = 16 + (int64_t)kLanesPerRow * V * 12;  // ClStatus<V>::kBytes
  return 256 + tiles * rec;
}

cudaError_t launch_cl(const ClArgs& a) {
  switch (a.dtype) {
    case kF32:
      return launch_cl_dtype<float>(a);
    case kF16:
      return launch_cl_dtype<__half>(a);
    case kBF16:
      return launch_cl_dtype<__nv_bfloat16>(a);
    default:
      return cudaErrorInvalidValue;
  }
}

}  // namespace fpscan
