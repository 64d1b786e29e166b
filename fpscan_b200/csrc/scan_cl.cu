// Channel-last scan: forward / reverse scan and fused backward on
// (batch, seqlen, dim) tensors, recurrence along the middle axis, sm_100a.
//
// The reference scans only the last axis; its README (README.md:94-99) has
// channel-last callers transpose with .mT.contiguous() before and after the
// call -- four extra passes over memory.  Here the scan runs on the
// channel-last tensor in place of those passes.
//
// One kernel, scan_cl_stream_kernel: a CTA streams a column of 8 channel
// vectors (128-byte rows) through a TMA tensor-tile ring (details below).
// With enough columns to fill the GPU each CTA takes a whole column.  With
// few columns the time axis is cut into segments, one CTA each, in three
// launches: a reduce pass (each segment's per-channel map), a small kernel
// composing the maps along each column (each segment's entering state), and
// a scan pass entering every segment with its state -- no inter-CTA waits.
//
// Head (zero initial state, gate ignored as at csrc/full_scan/full_scan.cu:96):
// timestep 0 (forward) or L-1 (reverse scan and backward).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>

#include "common.cuh"
#include "internal.h"

namespace fpscan {

namespace {

enum ClMode : int { kClFwd = 0, kClRev = 1, kClBwd = 2 };

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

// ------------------------------------------------------------------ streaming
// Column-streaming channel-last kernel: a CTA takes a column of kStreamVecs
// 16-byte channel vectors (128-byte rows) -- or one time segment of it --
// streamed chunk by chunk through an S-deep
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
  int64_t nseg;  // time segments per column (1: the whole column per CTA)
  int64_t cps;   // chunks per segment
  int64_t n_el;  // elements of each tensor (bounds checks of debug builds)
  int64_t n_map; // seg_map entries (bounds checks of debug builds)
  float2* seg_map;          // SPLIT 1: per (column, segment, vector, channel) map (A, B)
  const float* seg_carry;   // SPLIT 2: state entering each segment (same indexing)
};

// SPLIT (few columns: the time axis is cut into nseg segments, one CTA each):
//   0 -- the whole column (nseg = 1);
//   1 -- reduce: no output; the segment's map per channel (A = product of
//        its gates, B = its last state from a zero entering state) goes to
//        seg_map;
//   2 -- scan: as 0 within the segment, entering with seg_carry (segments
//        after the first; cl_seg_carry_kernel composes the maps in between).
template <typename T, int MODE, int TW, int S, int NTH, int SPLIT = 0>
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
  const int64_t col = (int64_t)blockIdx.x / p.nseg;
  const int64_t seg = (int64_t)blockIdx.x - col * p.nseg;  // processing order
  const int64_t b = col / p.cb, cblk = col - b * p.cb;
  const int64_t L = p.L;
  const int64_t head_t = DESC ? L - 1 : 0;
  const int64_t nck = (L + R - 1) / R;
  const int64_t k0 = seg * p.cps;                 // first chunk (processing order)
  const int64_t nloc = min(p.cps, nck - k0);      // chunks of this segment
  if (nloc <= 0) return;
  const int64_t cv = cblk * kStreamVecs + vec;
  const bool lane_ok = cv < p.dv;
  const bool aligned = (smem_addr(csm) & 127u) == 0;  // TMA destination rule, checked

  if (tid == 0) {
#pragma unroll
    for (int s = 0; s < S; ++s) mbar_init(&s_bar[s], 1);
    fence_mbar_init();
  }
  __syncthreads();
  pdl_wait();  // the previous kernel in the stream is complete from here on
  pdl_launch_dependents();
  if (!aligned) {
    if (tid == 0) atomicOr(&g_status, kStatusMisaligned);
    return;
  }

  const int x = (int)(cblk * kStreamVecs * V);
  int64_t issued = 0;  // local chunk index
  auto issue = [&](int64_t j) {
    const int64_t k = k0 + j;
    const int64_t m = DESC ? nck - 1 - k : k;
    const int s = (int)(j % S);
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
    for (; issued < min((int64_t)S, nloc); ++issued) issue(issued);

  T* out = static_cast<T*>(p.out);
  T* out2 = static_cast<T*>(p.out2);
  const int64_t row_elems = p.dv * V;
  const int64_t base = (b * L) * row_elems + cv * V;

  float seg_a[V];  // SPLIT 1: product of the segment's gates (thread group NG-1)
#pragma unroll
  for (int c = 0; c < V; ++c) seg_a[c] = 1.f;
  float st[V];     // state after the thread's last timestep
  int64_t j = 0;
  int s = 0;
  uint32_t phase = 0;
  bool aborted = false;
  for (; j < nloc; ++j) {
    const int64_t k = k0 + j;
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
    const int buf = (int)(j & 1);
    if (grp == 32 / kStreamVecs - 1)
#pragma unroll
      for (int c = 0; c < V; ++c) s_wt[buf][warp][c][vec] = make_float2(A[c], B[c]);

    if (__syncthreads_or(!ok)) {
      aborted = true;
      break;
    }
    // Pass 2 below still reads stage s, but every thread has finished the
    // previous chunk: refill that chunk's stage (issued == k - 1 + S).
    if (tid == 0 && j >= 1 && issued < nloc) {
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
    // (A segment's reduce pass also enters with exactly 0; a scan pass's
    // later segments enter with their carry.)
    bool zero = j == 0 && (seg == 0 || SPLIT == 1);
    if (j == 0) {
      const float* cin = p.seg_carry + ((col * p.nseg + seg) * kStreamVecs + vec) * V;
#pragma unroll
      for (int c = 0; c < V; ++c) st[c] = (SPLIT == 2 && seg > 0) ? cin[c] : 0.f;
    } else {
#pragma unroll
      for (int c = 0; c < V; ++c) st[c] = s_carry[buf ^ 1][vec][c];
    }
    if (SPLIT == 1 && tg == Cfg::NG - 1) {  // the chunk's gate product
      for (int q = 0; q < NW; ++q)
#pragma unroll
        for (int c = 0; c < V; ++c) seg_a[c] *= s_wt[buf][q][c][vec].x;
    }
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
      if (SPLIT != 1 && t >= 0 && t < L && lane_ok) {
        FPSCAN_DEBUG_ONLY(if (in_bounds(out + base + t * row_elems, 16, out, out + p.n_el)))
        *reinterpret_cast<uint4*>(out + base + t * row_elems) = pack_vec<T>(st);
        if (BWD) {
          float yp[V], dg[V];
          unpack<T>(s_c[lr * kStreamVecs + vec], yp);
#pragma unroll
          for (int c = 0; c < V; ++c) dg[c] = st[c] * yp[c];
          FPSCAN_DEBUG_ONLY(if (in_bounds(out2 + base + t * row_elems, 16, out2, out2 + p.n_el)))
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
    for (int64_t jj = j; jj < issued; ++jj)
      mbar_wait_bounded(&s_bar[jj % S], (uint32_t)((jj / S) & 1));
  }
  if (SPLIT == 1 && !aborted && tg == Cfg::NG - 1 && lane_ok) {
    float2* o = p.seg_map + ((col * p.nseg + seg) * kStreamVecs + vec) * V;
    FPSCAN_DEBUG_ONLY(if (in_bounds<8>(o, V * 8, p.seg_map, p.seg_map + p.n_map)))
#pragma unroll
    for (int c = 0; c < V; ++c) o[c] = make_float2(seg_a[c], st[c]);
  }
}

// Entering state of every segment after the first, per (column, vector,
// channel): the first segment's map holds its last state (it starts at the
// head); later ones compose A * state + B.
struct CarryArgs {
  const float2* seg_map;
  float* seg_carry;
  int64_t chans, ncol, nseg;
};

__global__ void cl_seg_carry_kernel(const CarryArgs ca) {
  const float2* __restrict__ seg_map = ca.seg_map;
  float* __restrict__ seg_carry = ca.seg_carry;
  const int64_t chans = ca.chans, ncol = ca.ncol, nseg = ca.nseg;
  pdl_wait();
  pdl_launch_dependents();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= ncol * chans) return;
  const int64_t col = i / chans, ch = i - col * chans;
  float state = 0.f;
  for (int64_t sg = 0; sg + 1 < nseg; ++sg) {
    const float2 m = seg_map[(col * nseg + sg) * chans + ch];
    state = sg == 0 ? m.y : fmaf(m.x, state, m.y);
    seg_carry[(col * nseg + sg + 1) * chans + ch] = state;
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
                     int64_t dim, int ts, int row_bytes) {
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

// Few-column plan: time segments per column so that columns x segments is
// about two CTAs per SM, each segment at least two chunks.  FPSCAN_B200_CL_PATH
// =stream / =split forces one CTA per column / the segmented path.
constexpr int64_t kStreamMinCols = 128;

int num_sms_or_default() {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
    return 148;
  return sms;
}

int cl_force() {
  static const int force = [] {
    const char* v = getenv("FPSCAN_B200_CL_PATH");
    if (v && !strcmp(v, "stream")) return 1;
    if (v && !strcmp(v, "split")) return 2;
    return 0;
  }();
  return force;
}

int64_t cl_columns(int64_t batch, int64_t dim, int dtype) {
  const int64_t dv = dim / (16 / dtype_size(dtype));
  return batch * ((dv + kStreamVecs - 1) / kStreamVecs);
}

// Upper bound of segments per column (the workspace is sized for it).
int64_t cl_max_segments(int64_t cols) {
  if (cl_force() == 1 || (cl_force() == 0 && cols >= kStreamMinCols)) return 1;
  const int64_t want = (2 * (int64_t)num_sms_or_default() + cols - 1) / cols;
  return std::max<int64_t>(want, 2);
}

struct SegPlan {
  int64_t nseg, cps;
};
SegPlan cl_seg_plan(int64_t cols, int64_t seqlen, int64_t R) {
  const int64_t nck = (seqlen + R - 1) / R;
  const int64_t want = cl_max_segments(cols);
  if (want <= 1 || nck < 4) return {1, nck};
  const int64_t cps = std::max<int64_t>(2, (nck + want - 1) / want);
  return {(nck + cps - 1) / cps, cps};
}

template <typename Kern>
cudaError_t configure(Kern kern, int smem, int* configured) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) configured[dev] = 1;
  }
  return cudaSuccess;
}

template <typename T, int MODE, int TW, int S, int NTH = kThreads>
cudaError_t launch_stream_t(const ClArgs& a) {
  using Cfg = StreamCfg<T, MODE, TW, S, NTH>;
  constexpr int V = Elem<T>::kVec;
  constexpr int smem = Cfg::smem();
  static int conf0[64] = {0}, conf1[64] = {0}, conf2[64] = {0};
  // Bind the device's primary context to this thread before encoding the
  // tensor maps: cuTensorMapEncodeTiled checks the addresses against the
  // current context, and a thread that has made no runtime call yet (e.g.
  // autograd's backward worker) has none.
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaSetDevice(dev);
  if (e != cudaSuccess) return e;
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
  const SegPlan plan = cl_seg_plan(cols, a.seqlen, R);
  p.nseg = plan.nseg;
  p.cps = plan.cps;
  p.n_el = a.batch * a.seqlen * a.dim;
  if (plan.nseg == 1) {
    auto kern = scan_cl_stream_kernel<T, MODE, TW, S, NTH, 0>;
    if ((e = configure(kern, smem, conf0)) != cudaSuccess) return e;
    return launch_pdl(kern, (unsigned)cols, NTH, smem, a.stream, p);
  }
  // segmented: reduce, compose, scan
  const int64_t chans = (int64_t)kStreamVecs * V;
  const int64_t n = cols * plan.nseg * chans;
  const int64_t map_bytes = (n * 8 + 255) / 256 * 256;
  if ((int64_t)a.workspace_bytes < map_bytes + n * 4) return cudaErrorInvalidValue;
  p.seg_map = static_cast<float2*>(a.workspace);
  p.n_map = n;
  p.seg_carry = reinterpret_cast<const float*>(static_cast<char*>(a.workspace) + map_bytes);
  const unsigned grid = (unsigned)(cols * plan.nseg);
  auto k1 = scan_cl_stream_kernel<T, MODE, TW, S, NTH, 1>;
  auto k2 = scan_cl_stream_kernel<T, MODE, TW, S, NTH, 2>;
  if ((e = configure(k1, smem, conf1)) != cudaSuccess) return e;
  if ((e = configure(k2, smem, conf2)) != cudaSuccess) return e;
  if ((e = launch_pdl(k1, grid, NTH, smem, a.stream, p)) != cudaSuccess) return e;
  const int64_t threads = cols * chans;
  CarryArgs ca{p.seg_map, const_cast<float*>(p.seg_carry), chans, cols, plan.nseg};
  if ((e = launch_pdl(cl_seg_carry_kernel, (unsigned)((threads + 255) / 256), 256, 0, a.stream,
                      ca)) != cudaSuccess)
    return e;
  return launch_pdl(k2, grid, NTH, smem, a.stream, p);
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
  if (a.backward) return launch_stream_mode<T, kClBwd>(a);
  return a.reverse ? launch_stream_mode<T, kClRev>(a) : launch_stream_mode<T, kClFwd>(a);
}

}  // namespace

int64_t cl_workspace_bytes(int64_t batch, int64_t seqlen, int64_t dim, int dtype, bool backward) {
  (void)seqlen;
  (void)backward;
  const int64_t cols = cl_columns(batch, dim, dtype);
  const int64_t nseg = cl_max_segments(cols);
  if (nseg <= 1) return 256;
  const int64_t n = cols * nseg * kStreamVecs * (16 / dtype_size(dtype));
  return (n * 8 + 255) / 256 * 256 + n * 4;
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
