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

#include <atomic>
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

template <typename T, int MODE, int TS>
struct ClCfg {
  static constexpr int kTiles = MODE == kClBwd ? 3 : 2;
  static constexpr int V = Elem<T>::kVec;
  static constexpr int kTileBytes = TS * kRowBytes;
  static constexpr int kTotBytes = kWarps * kLanesPerRow * V * 8;  // per-warp maps
  static constexpr int kCarryBytes = kLanesPerRow * V * 4;
  // + 128: the base is rounded up to the 128-byte alignment TMA tensor
  // copies require (dynamic shared memory follows the static variables)
  static constexpr int smem() { return kTiles * kTileBytes + kTotBytes + kCarryBytes + 128; }
};

template <typename T, int MODE, int TS>
__global__ void __launch_bounds__(kThreads, 2) scan_cl_kernel(const __grid_constant__ ClParams p) {
  using Cfg = ClCfg<T, MODE, TS>;
  constexpr int V = Elem<T>::kVec;
  constexpr int TW = TS / kWarps;  // timesteps per warp
  constexpr bool DESC = MODE != kClFwd;
  constexpr bool BWD = MODE == kClBwd;
  using St = ClStatus<V>;
  static_assert(TS % kWarps == 0, "TS must be a multiple of the warp count");

  extern __shared__ __align__(128) unsigned char csm_raw[];
  unsigned char* csm = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(csm_raw) + 127) & ~uintptr_t(127));
  const uint4* s_a = reinterpret_cast<const uint4*>(csm);
  const uint4* s_b = reinterpret_cast<const uint4*>(csm + Cfg::kTileBytes);
  const uint4* s_c = reinterpret_cast<const uint4*>(csm + 2 * Cfg::kTileBytes);
  float2* s_tot = reinterpret_cast<float2*>(csm + Cfg::kTiles * Cfg::kTileBytes);  // [8][32][V]
  float* s_carry = reinterpret_cast<float*>(csm + Cfg::kTiles * Cfg::kTileBytes + Cfg::kTotBytes);
  __shared__ __align__(8) uint64_t s_bar;
  __shared__ long long s_ticket;
  __shared__ int s_hf[kWarps];

  const int tid = threadIdx.x, lane = tid & 31, pw = tid >> 5;  // pw: warp in processing order

  if (tid == 0) {
    s_ticket = (long long)atomicAdd(p.counter, 1ull);
    mbar_init(&s_bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  const int64_t ticket = s_ticket;
  if (ticket >= p.ncol * p.segs) return;
  const int64_t seg_p = ticket / p.ncol;  // segment in processing order
  const int64_t col = ticket - seg_p * p.ncol;
  const int64_t b = col / p.cb, cblk = col - b * p.cb;
  const int64_t seg_m = DESC ? p.segs - 1 - seg_p : seg_p;
  const int64_t s0 = seg_m * TS;  // first timestep of the tile
  const int64_t L = p.L;
  const int64_t head_t = DESC ? L - 1 : 0;
  const int64_t cv = cblk * kLanesPerRow + lane;  // this lane's channel vector
  const bool lane_ok = cv < p.dv;

  // TMA tensor copies need a 128-byte aligned destination: checked, never
  // assumed (a failed check aborts the tile like a copy that never lands)
  const bool aligned = (smem_addr(csm) & 127u) == 0;
  if (tid == 0 && !aligned) atomicOr(&g_status, kStatusMisaligned);
  if (tid == 0 && aligned) {
    const int x = (int)(cblk * kLanesPerRow * V);
    mbar_expect_tx(&s_bar, (uint32_t)(Cfg::kTiles * Cfg::kTileBytes));
    if (BWD) {
      tma_load_3d(csm, &p.tm_a, x, (int)(s0 + 1), (int)b, &s_bar);
      tma_load_3d(csm + Cfg::kTileBytes, &p.tm_b, x, (int)s0, (int)b, &s_bar);
      tma_load_3d(csm + 2 * Cfg::kTileBytes, &p.tm_c, x, (int)(s0 - 1), (int)b, &s_bar);
    } else {
      tma_load_3d(csm, &p.tm_a, x, (int)s0, (int)b, &s_bar);
      tma_load_3d(csm + Cfg::kTileBytes, &p.tm_b, x, (int)s0, (int)b, &s_bar);
    }
  }
  // uniform across the CTA: a copy that never lands aborts every thread
  const bool ok = __syncthreads_and(aligned && mbar_wait_bounded(&s_bar, 0));

  // ---- pass 1: the thread's map over its TW timesteps, per channel
  float A[V], B[V];
  bool hf = false;
  if (ok) {
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
  } else {
#pragma unroll
    for (int c = 0; c < V; ++c) {
      A[c] = 1.f;
      B[c] = 0.f;
    }
  }
#pragma unroll
  for (int c = 0; c < V; ++c) s_tot[(pw * kLanesPerRow + lane) * V + c] = make_float2(A[c], B[c]);
  if (lane == 0) s_hf[pw] = hf ? 1 : 0;
  __syncthreads();

  // ---- exclusive prefix over the earlier warps (processing order)
  float EA[V], EB[V];
  bool have = false, ef = false;
  {
    int q0 = 0;
    for (int q = 0; q < pw; ++q)
      if (s_hf[q]) {
        q0 = q;
        ef = true;
      }
    for (int q = q0; q < pw; ++q) {
      const float2* t = s_tot + (q * kLanesPerRow + lane) * V;
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
  }

  // ---- look-back (last warp in processing order): publish, find the carry
  if (pw == kWarps - 1) {
    float GA[V], GB[V];
    bool gf;
    if (hf || !have) {
      gf = hf;
#pragma unroll
      for (int c = 0; c < V; ++c) {
        GA[c] = A[c];
        GB[c] = B[c];
      }
    } else {
      gf = ef;
#pragma unroll
      for (int c = 0; c < V; ++c) {
        GA[c] = EA[c] * A[c];
        GB[c] = fmaf(EB[c], A[c], B[c]);
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
          *reinterpret_cast<float4*>(incl + c) = make_float4(src_b[c], src_b[c + 1], src_b[c + 2], src_b[c + 3]);
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

    if (gf || seg_p == 0 || !ok) {
      // The tile holds the head (or is the first one): its inclusive state
      // does not depend on any carry.
      publish(GA, GB, true);
    } else {
      const unsigned char* prev = p.status + (ticket - p.ncol) * (int64_t)St::kBytes;
      const uint32_t f0 = ld_acquire_u32(reinterpret_cast<const uint32_t*>(prev));
      const bool direct = __all_sync(0xffffffffu, f0 == incl_flag);
      if (!direct) publish(GA, GB, false);
      // acc: composition of the tiles between the found one and this one
      float acc_a[V], acc_b[V];
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
            for (int k = 0; k < 4; ++k)
              carry[c + k] = acc_have ? fmaf(acc_a[c + k], vv[k], acc_b[c + k]) : vv[k];
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
#pragma unroll
    for (int c = 0; c < V; ++c) s_carry[lane * V + c] = carry[c];
  }
  __syncthreads();
  if (!ok) {
    if (tid == 0 && aligned) mbar_wait_bounded(&s_bar, 0);  // let a late copy land before exit
    return;
  }

  // ---- pass 2: rerun the recurrence from the thread's entering state
  float st[V];
#pragma unroll
  for (int c = 0; c < V; ++c) {
    const float cin = s_carry[lane * V + c];
    st[c] = ef ? EB[c] : (have ? fmaf(EA[c], cin, EB[c]) : cin);
  }
  T* out = static_cast<T*>(p.out);
  T* out2 = static_cast<T*>(p.out2);
  const int64_t row_elems = p.dv * V;
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
      uint4* dst = reinterpret_cast<uint4*>(out + base + t * row_elems);
      *dst = pack_vec<T>(st);
      if (BWD) {
        float yp[V], dg[V];
        unpack<T>(s_c[lr * kLanesPerRow + lane], yp);
#pragma unroll
        for (int c = 0; c < V; ++c) dg[c] = st[c] * yp[c];
        *reinterpret_cast<uint4*>(out2 + base + t * row_elems) = pack_vec<T>(dg);
      }
    }
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

// 3-D map over (dim, seqlen, batch) with a (32 vectors, TS, 1) box.
cudaError_t make_map(CUtensorMap* m, const void* ptr, int dtype, int64_t batch, int64_t L,
                     int64_t dim, int ts) {
  auto fn = encode_fn();
  if (!fn) return cudaErrorNotSupported;
  const int es = dtype_size(dtype);
  const CUtensorMapDataType dt = dtype == kF32   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : dtype == kF16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const cuuint64_t dims[3] = {(cuuint64_t)dim, (cuuint64_t)L, (cuuint64_t)batch};
  const cuuint64_t strides[2] = {(cuuint64_t)(dim * es), (cuuint64_t)(L * dim * es)};
  const cuuint32_t box[3] = {(cuuint32_t)(kRowBytes / es), (cuuint32_t)ts, 1};
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

template <typename T, int MODE>
constexpr int cl_ts() {
  return MODE == kClBwd ? 32 : 64;
}

template <typename T, int MODE>
cudaError_t launch_cl_t(const ClArgs& a) {
  constexpr int TS = cl_ts<T, MODE>();
  constexpr int V = Elem<T>::kVec;
  constexpr int smem = ClCfg<T, MODE, TS>::smem();
  auto kern = scan_cl_kernel<T, MODE, TS>;
  static int configured[64] = {0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) configured[dev] = 1;
  }
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
  kern<<<(unsigned)tiles, kThreads, smem, a.stream>>>(p);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_cl_dtype(const ClArgs& a) {
  if (a.backward) return launch_cl_t<T, kClBwd>(a);
  return a.reverse ? launch_cl_t<T, kClRev>(a) : launch_cl_t<T, kClFwd>(a);
}

}  // namespace

int64_t cl_workspace_bytes(int64_t batch, int64_t seqlen, int64_t dim, int dtype, bool backward) {
  const int es = dtype_size(dtype);
  const int V = 16 / es;
  const int ts = backward ? 32 : 64;  // cl_ts<>
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
