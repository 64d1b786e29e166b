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

  // Stage the whole segment at once: chunk c (processing order) -> buffer c.
  if (tid == 0) {
    const uint32_t bytes = (uint32_t)(CH * sizeof(T));
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int64_t off = (int64_t)(REV ? NC - 1 - c : c) << LGCH;
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
    SegStatus* st = p.status + t;
    const uint32_t agg_flag = p.epoch << 1, incl_flag = (p.epoch << 1) | 1u;
    float state_in = 0.f;
    if (sp == 0) {
      st->b_incl = agg_b;  // zero initial state, first gate ignored: the final state
      st_release(&st->flag, incl_flag);
    } else {
      st->a = agg_a;
      st->b = agg_b;
      st_release(&st->flag, agg_flag);
      float acc_a = 1.f, acc_b = 0.f;  // composition of the segments after j, before t
      const uint64_t t0 = global_ns();
      for (int64_t j = t - 1;; --j) {
        const SegStatus* sj = p.status + j;
        uint32_t f;
        uint32_t spins = 0;
        bool timed_out = false;
        while (true) {
          f = ld_acquire(&sj->flag);
          if ((f >> 1) == p.epoch) break;
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
    }
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
#pragma unroll
    for (int k2 = 0; k2 < NV; ++k2) dst[k2] = pack_vec<T>(f + k2 * V);
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
  kern<<<(unsigned)tiles, kThreads, kSplitSmem, a.stream>>>(p);
  return cudaGetLastError();
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
