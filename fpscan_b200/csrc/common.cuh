// Shared device helpers for the fpscan B200 kernels (sm_100a only).
//
// The scan operator is the first-order linear recurrence
//     y[t] = g[t] * y[t-1] + x[t]
// represented as affine maps (A, B): y -> A*y + B.  Composing an earlier map
// (Ap, Bp) with a later one (A, B) gives (Ap*A, Bp*A + B); the scan of x over
// g is the B component of the inclusive prefix composition.  All arithmetic
// is fp32 regardless of the storage type, as in the reference kernel
// (csrc/full_scan/full_scan.cu:87-111 accumulates in float).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>

namespace fpscan {

// Threads per CTA of every streaming kernel.  Each thread owns NV
// consecutive 16-byte vectors of a chunk (NV = 1 or 2, a kernel template
// parameter), so a chunk is kThreads * NV * 16 bytes per tensor.
constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

// Device-side status word.  Bounded waits that give up set a bit here instead
// of hanging the GPU; the host reads and clears it through
// fpscan_device_status().
enum : unsigned {
  kStatusWaitTimeout = 1u,
  kStatusLookbackTimeout = 2u,
  kStatusMisaligned = 4u,
  kStatusLinkTimeout = 8u,
  kStatusBounds = 16u,
};

extern __device__ unsigned int g_status;

// Limit of every bounded wait, in ns of %globaltimer (per device; default
// 2 s; fpscan_set_wait_limit_ns).  Read only once a wait did not complete
// at its first try.
extern __device__ unsigned long long g_wait_limit_ns;

// ---------------------------------------------------------------- conversion
template <typename T> struct Elem;
template <> struct Elem<float> {
  static constexpr int kVec = 4;
  __device__ __forceinline__ static float load(float v) { return v; }
  __device__ __forceinline__ static float store(float v) { return v; }
};
template <> struct Elem<__half> {
  static constexpr int kVec = 8;
  __device__ __forceinline__ static float load(__half v) { return __half2float(v); }
  __device__ __forceinline__ static __half store(float v) { return __float2half_rn(v); }
};
template <> struct Elem<__nv_bfloat16> {
  static constexpr int kVec = 8;
  __device__ __forceinline__ static float load(__nv_bfloat16 v) { return __bfloat162float(v); }
  __device__ __forceinline__ static __nv_bfloat16 store(float v) { return __float2bfloat16_rn(v); }
};

// One 16-byte vector viewed as kVec elements.
template <typename T> union Vec16 {
  uint4 raw;
  T e[Elem<T>::kVec];
};

// ---------------------------------------------------------------- mbarrier / bulk copy
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

// Plain arrive (no transaction bytes): completes the barrier's phase by
// itself (count 1).  Used to hand consumers an end-of-work marker through a
// stage that receives no copy.
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// Non-multicast 1-D bulk copy global -> shared, completing on `bar`.
// Both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// Debug builds (-DFPSCAN_DEBUG_BOUNDS: libfpscan_b200_debug.so, built by
// fpscan_b200.build.build_debug) check every global access that a kernel
// computes itself -- bulk-copy sources, direct loads, output stores, carry
// arrays -- against the extent [lo, hi) of the tensor it belongs to and the
// access's alignment; an access outside is skipped and recorded as
// kStatusBounds, so a wrong index shows up as a status bit instead of a
// fault or a silent write elsewhere.  The checks sit inside
// FPSCAN_DEBUG_ONLY(...), which release builds drop, so the release kernels
// are compiled from unchanged code (same registers, same schedule).
#ifdef FPSCAN_DEBUG_BOUNDS
#define FPSCAN_DEBUG_ONLY(...) __VA_ARGS__
#else
#define FPSCAN_DEBUG_ONLY(...)
#endif

template <int ALIGN = 16>
__device__ __forceinline__ bool in_bounds(const void* p, uint64_t bytes, const void* lo,
                                          const void* hi) {
  const char* c = static_cast<const char*>(p);
  const bool ok = c >= static_cast<const char*>(lo) && c + bytes <= static_cast<const char*>(hi) &&
                  (reinterpret_cast<uintptr_t>(c) % ALIGN) == 0;
  if (!ok) atomicOr(&g_status, kStatusBounds);
  return ok;
}

// Programmatic dependent launch.  A kernel launched with the programmatic
// stream serialization attribute may start while the previous kernel in its
// stream is still running; pdl_wait() blocks until that kernel has completed
// and its memory operations are visible (a no-op without the attribute).
// Every thread calls it before its first global access.  pdl_launch_dependents()
// lets the next such kernel start its own prologue early.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Wait for phase `parity` of `bar`, giving up after g_wait_limit_ns of wall
// time.  A bulk copy from valid device memory always completes, so the limit
// only guards against a fault elsewhere turning into a hung GPU.  Returns
// false on timeout (and records it in g_status).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  const uint64_t limit = *(volatile unsigned long long*)&g_wait_limit_ns;
  for (uint32_t it = 0;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 255u && global_ns() - t0 > limit) {
      atomicOr(&g_status, kStatusWaitTimeout);
      return false;
    }
  }
}

// ---------------------------------------------------------------- rank links
// Cross-GPU hand-off of per-row values over NVLink peer memory (chained
// sequence sharding).  A value travels with its epoch in one 64-bit word
// (epoch << 32 | float bits) written by one single-copy-atomic relaxed store,
// so the consumer polls the word itself: no flag, no fence.  Acks (the epoch
// a consumer has taken) are relaxed 32-bit stores issued after the value was
// loaded and used.  Loads are issued early (a chunk's start) and completed
// late, so a poll that finds the word ready costs no stall.
__device__ __forceinline__ uint64_t ld_relaxed_sys_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ void st_relaxed_sys_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_relaxed_sys_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ void st_relaxed_sys_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint64_t link_word(float v, uint32_t epoch) {
  return ((uint64_t)epoch << 32) | __float_as_uint(v);
}

// Completes a poll of the link word at p begun with `first` (an earlier load
// of p): re-polls until its epoch reaches `epoch` (wrap-safe), bounded by
// g_wait_limit_ns, then returns the value.  On timeout it records
// kStatusLinkTimeout and returns NaN, so the rows that needed the value come
// out visibly wrong (NaN) rather than plausible.
__device__ __forceinline__ float link_take(const uint64_t* p, uint32_t epoch, uint64_t first) {
  uint64_t w = first;
  if ((int)((uint32_t)(w >> 32) - epoch) < 0) {
    const uint64_t t0 = global_ns();
    const uint64_t limit = *(volatile unsigned long long*)&g_wait_limit_ns;
    for (uint32_t it = 0;; ++it) {
      w = ld_relaxed_sys_u64(p);
      if ((int)((uint32_t)(w >> 32) - epoch) >= 0) break;
      if ((it & 63u) == 63u && global_ns() - t0 > limit) {
        atomicOr(&g_status, kStatusLinkTimeout);
        return __int_as_float(0x7fc00000);
      }
    }
  }
  return __uint_as_float((uint32_t)w);
}

// Completes a wait, begun with `first`, for the 32-bit word at p to reach
// `target` (wrap-safe); bounded like link_take.
__device__ __forceinline__ void link_wait_ack(const uint32_t* p, uint32_t target, uint32_t first) {
  if ((int)(first - target) >= 0) return;
  const uint64_t t0 = global_ns();
  const uint64_t limit = *(volatile unsigned long long*)&g_wait_limit_ns;
  for (uint32_t it = 0;; ++it) {
    if ((int)(ld_relaxed_sys_u32(p) - target) >= 0) return;
    if ((it & 63u) == 63u && global_ns() - t0 > limit) {
      atomicOr(&g_status, kStatusLinkTimeout);
      return;
    }
  }
}

// ---------------------------------------------------------------- scan combine
// Inclusive Hillis-Steele scan of (A, B) pairs across `width` lanes
// (width a power of two <= 32, segments aligned to multiples of width).
__device__ __forceinline__ void warp_scan_pair(float& a, float& b, int lane, int width) {
  const int seg_lane = lane & (width - 1);
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    if (d >= width) break;
    const float pa = __shfl_up_sync(0xffffffffu, a, d);
    const float pb = __shfl_up_sync(0xffffffffu, b, d);
    if (seg_lane >= d) {
      b = fmaf(pb, a, b);
      a = pa * a;
    }
  }
}

// Exclusive per-thread prefix within warp segments of `width` lanes, from
// the thread's own total (ta, tb): inclusive Hillis-Steele scan, then a
// shift by one lane.  Leaves the inclusive value in (ta, tb).
__device__ __forceinline__ void warp_exclusive(float& ta, float& tb, int lane, int width,
                                               float& ea, float& eb) {
  warp_scan_pair(ta, tb, lane, width);
  ea = __shfl_up_sync(0xffffffffu, ta, 1);
  eb = __shfl_up_sync(0xffffffffu, tb, 1);
  if ((lane & (width - 1)) == 0) {
    ea = 1.f;
    eb = 0.f;
  }
}

// Block-level step after the warp scans.  Every warp redundantly scans the
// kWarps warp totals across its lanes 0..kWarps-1 (segmented in groups of
// `seg_warps` warps), so no second barrier is needed.
//   (pa, pb): in = the thread's exclusive prefix within its warp segment,
//             out = its exclusive prefix within its segment of seg_warps warps;
//   (ca, cb): the composition of all kWarps totals (the chunk total when one
//             segment spans the CTA, i.e. seg_warps == kWarps).
// Compositions start from real operands, never from an identity, so a
// non-finite A (e.g. an ignored first gate) never meets a 0.
__device__ __forceinline__ void compose_warp_totals(const float2* wt, int lane, int warp,
                                                    int seg_warps, float& pa, float& pb,
                                                    float& ca, float& cb) {
  float2 t = wt[lane & (kWarps - 1)];
  const int sl = lane & (seg_warps - 1);
#pragma unroll
  for (int d = 1; d < kWarps; d <<= 1) {
    if (d >= seg_warps) break;
    const float qa = __shfl_up_sync(0xffffffffu, t.x, d);
    const float qb = __shfl_up_sync(0xffffffffu, t.y, d);
    if (sl >= d) {
      t.y = fmaf(qb, t.x, t.y);
      t.x = qa * t.x;
    }
  }
  const float wa = __shfl_sync(0xffffffffu, t.x, (warp - 1) & (kWarps - 1));
  const float wb = __shfl_sync(0xffffffffu, t.y, (warp - 1) & (kWarps - 1));
  ca = __shfl_sync(0xffffffffu, t.x, kWarps - 1);
  cb = __shfl_sync(0xffffffffu, t.y, kWarps - 1);
  if ((warp & (seg_warps - 1)) != 0) {
    pb = fmaf(wb, pa, pb);
    pa = wa * pa;
  }
}

// Loads a thread's NV consecutive 16-byte vectors from shared memory.
// (A bank-conflict-free swizzled order was measured slower: the selects it
// needs cost more issue slots than the 2-way conflicts of this order.)
template <int NV>
__device__ __forceinline__ void lds_vecs(const uint4* src, uint4 (&r)[NV]) {
#pragma unroll
  for (int q = 0; q < NV; ++q) r[q] = src[q];
}

// Packs fp32 values into one 16-byte vector of T with paired conversions
// (one cvt for two half values).
template <typename T>
__device__ __forceinline__ uint4 pack_vec(const float* v);
template <>
__device__ __forceinline__ uint4 pack_vec<float>(const float* v) {
  return make_uint4(__float_as_uint(v[0]), __float_as_uint(v[1]), __float_as_uint(v[2]),
                    __float_as_uint(v[3]));
}
template <>
__device__ __forceinline__ uint4 pack_vec<__nv_bfloat16>(const float* v) {
  uint4 r;
  uint32_t* w = reinterpret_cast<uint32_t*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t*>(&h);
  }
  return r;
}
template <>
__device__ __forceinline__ uint4 pack_vec<__half>(const float* v) {
  uint4 r;
  uint32_t* w = reinterpret_cast<uint32_t*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 h = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t*>(&h);
  }
  return r;
}

// Gate activations fused into the loads: the kernels read pre-activation
// values z and use g = act(z), computed in fp32.  exp(-softplus(z)) =
// 1 / (1 + e^z) is the sigmoid of -z.  act_grad gives dg/dz from g.
enum Act : int { kActNone = 0, kActSigmoid = 1, kActExpNegSoftplus = 2, kActExp = 3 };

// Hardware tanh (one MUFU op; relative error about 2^-11).
__device__ __forceinline__ float tanh_approx(float x) {
  float r;
  asm("tanh.approx.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// For fp32 data the sigmoids use the fast exp and divide intrinsics (a few
// ulp).  For fp16 / bf16 data, sigmoid(x) = 0.5 + 0.5 tanh(x / 2) costs one
// MUFU op; its error is well below the 2^-8 / 2^-11 rounding of the gate
// that an unfused producer would store in the input type.  (__fdividef
// returns 0 when the denominator overflows to inf, the correct limit.)
template <int ACT, typename T>
__device__ __forceinline__ float act_fwd(float z) {
  constexpr bool kHalf = sizeof(T) == 2;
  if constexpr (ACT == kActSigmoid) {
    if constexpr (kHalf) return fmaf(0.5f, tanh_approx(0.5f * z), 0.5f);
    else return __fdividef(1.f, 1.f + __expf(-z));
  } else if constexpr (ACT == kActExpNegSoftplus) {
    if constexpr (kHalf) return fmaf(-0.5f, tanh_approx(0.5f * z), 0.5f);
    else return __fdividef(1.f, 1.f + __expf(z));
  } else if constexpr (ACT == kActExp) {
    return __expf(z);
  } else {
    return z;
  }
}

template <int ACT>
__device__ __forceinline__ float act_grad(float g) {
  if constexpr (ACT == kActSigmoid) return g * (1.f - g);
  else if constexpr (ACT == kActExpNegSoftplus) return -g * (1.f - g);
  else if constexpr (ACT == kActExp) return g;
  else return 1.f;
}

constexpr int ilog2(int v) { return v <= 1 ? 0 : 1 + ilog2(v >> 1); }

}  // namespace fpscan
