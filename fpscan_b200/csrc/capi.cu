// C-ABI entry points (include/fpscan_b200.h): argument validation, dispatch
// and error reporting.  The reference performs its checks with TORCH_CHECK
// (csrc/full_scan/full_scan.h:7-15, csrc/full_scan/full_scan.cu:181-182,
// 232, 240-256); here the same conditions, plus the ones it omits (output
// shape/alignment, aliasing, launch errors), produce FPSCAN_ERR_* codes with a
// message in fpscan_last_error().
#include "../../include/fpscan_b200.h"
#include "common.cuh"
#include "internal.h"

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <cstdlib>
#include <string>

namespace fpscan {

__device__ unsigned int g_status = 0;
__device__ unsigned long long g_wait_limit_ns = 2000000000ull;

namespace {
// Reads and clears the status word into *dst (device or mapped host memory).
__global__ void status_take_kernel(unsigned* dst) { *dst = atomicExch(&g_status, 0u); }

// Bounds-checking builds: checks (without accessing it) an address one
// element past a 4-element extent, which records kStatusBounds.  Release
// builds: an empty kernel.
__global__ void bounds_probe_kernel() {
  FPSCAN_DEBUG_ONLY(__shared__ float extent[4]; in_bounds<4>(extent + 4, 4, extent, extent + 4);)
}
}  // namespace

namespace {

thread_local std::string t_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return code;
}

int ok() {
  t_last_error.clear();
  return FPSCAN_OK;
}

bool is_pow2(int64_t v) { return v > 0 && (v & (v - 1)) == 0; }

int num_sms_current() {
  static std::atomic<int> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev >= 0 && dev < 64) {
    int c = cache[dev].load(std::memory_order_relaxed);
    if (c > 0) return c;
  }
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
    sms = 148;
  if (dev >= 0 && dev < 64) cache[dev].store(sms, std::memory_order_relaxed);
  return sms;
}

// Counters of the dynamic row-unit scheduling (UnitSched, internal.h): one
// 32-bit word per launch, zero between launches (a launch's last claim
// resets its word), so launches that may run at the same time must not
// share one.  Live launches cycle through kRingSlots words per device (a word
// comes back only after kRingSlots later launches on that device); launches
// recorded into a CUDA graph keep a word of their own for good, since the
// graph can be replayed at any time (static tiling once those run out; two
// executable instances of one captured graph share its words and must not
// run at the same time).  The
// words are a file-scope device array, zeroed when the module loads on each
// device, so no call allocates or clears memory for them.
constexpr uint32_t kRingSlots = 1u << 16, kGraphSlots = 1u << 16;
__device__ unsigned g_unit_ctr[kRingSlots + kGraphSlots];

struct SchedPool {
  std::atomic<unsigned*> base{nullptr};
  std::atomic<uint32_t> ring{0};
  std::atomic<uint32_t> graph{0};
};
SchedPool g_sched[64];

unsigned* sched_counter(cudaStream_t stream) {
  static const bool off = getenv("FPSCAN_B200_STATIC_TILES") != nullptr;
  if (off) return nullptr;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cs) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  SchedPool& pool = g_sched[dev];
  unsigned* base = pool.base.load(std::memory_order_acquire);
  if (base == nullptr) {
    if (cs != cudaStreamCaptureStatusNone) return nullptr;  // resolve outside captures
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_unit_ctr) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    base = static_cast<unsigned*>(p);
    pool.base.store(base, std::memory_order_release);
  }
  if (cs == cudaStreamCaptureStatusNone)
    return base + pool.ring.fetch_add(1, std::memory_order_relaxed) % kRingSlots;
  const uint32_t g = pool.graph.fetch_add(1, std::memory_order_relaxed);
  return g < kGraphSlots ? base + kRingSlots + g : nullptr;
}

struct Span {
  const char* name;
  uintptr_t lo, hi;
};

bool overlaps(const Span& a, const Span& b) { return a.lo < b.hi && b.lo < a.hi; }

int check_dtype(int dtype) {
  if (dtype != kF32 && dtype != kF16 && dtype != kBF16)
    return fail(FPSCAN_ERR_INVALID,
                "unsupported dtype code %d: expecting float32 (0), float16 (1) or bfloat16 (2)",
                dtype);
  return FPSCAN_OK;
}

int check_ptr(const void* p, const char* name) {
  if (p == nullptr) return fail(FPSCAN_ERR_INVALID, "%s is NULL", name);
  if (reinterpret_cast<uintptr_t>(p) % 16 != 0)
    return fail(FPSCAN_ERR_INVALID, "%s must be 16-byte aligned", name);
  return FPSCAN_OK;
}

// rows = batch*dim, with overflow and sign checks.
int check_shape(int64_t batch, int64_t dim, int64_t seqlen, int64_t min_l, int64_t max_l,
                int64_t* rows) {
  if (batch < 0 || dim < 0)
    return fail(FPSCAN_ERR_INVALID, "batch (%lld) and dim (%lld) must be non-negative",
                (long long)batch, (long long)dim);
  if (!is_pow2(seqlen) || seqlen < min_l || seqlen > max_l)
    return fail(FPSCAN_ERR_INVALID, "seqlen must be a power of 2, >= %lld, <= %lld (got %lld)",
                (long long)min_l, (long long)max_l, (long long)seqlen);
  if (dim != 0 && batch > INT64_MAX / dim)
    return fail(FPSCAN_ERR_INVALID, "batch*dim overflows");
  const int64_t r = batch * dim;
  if (r != 0 && r > INT64_MAX / seqlen / 4)
    return fail(FPSCAN_ERR_INVALID, "tensor too large");
  if (r > (int64_t)0x7fffffff * 64)
    return fail(FPSCAN_ERR_INVALID, "batch*dim too large for the launch grid");
  *rows = r;
  return FPSCAN_OK;
}

// Shape check of the any-seqlen entry points: seqlen >= 1, no power-of-two
// or upper limit beyond what 64-bit offsets and the grid allow.
int check_shape_any(int64_t batch, int64_t dim, int64_t seqlen, int64_t* rows) {
  if (batch < 0 || dim < 0)
    return fail(FPSCAN_ERR_INVALID, "batch (%lld) and dim (%lld) must be non-negative",
                (long long)batch, (long long)dim);
  if (seqlen < 1) return fail(FPSCAN_ERR_INVALID, "seqlen must be >= 1 (got %lld)", (long long)seqlen);
  if (dim != 0 && batch > INT64_MAX / dim)
    return fail(FPSCAN_ERR_INVALID, "batch*dim overflows");
  const int64_t r = batch * dim;
  if (r != 0 && r > INT64_MAX / seqlen / 8)
    return fail(FPSCAN_ERR_INVALID, "tensor too large");
  if (r > (int64_t)0x7fffffff * 64)
    return fail(FPSCAN_ERR_INVALID, "batch*dim too large for the launch grid");
  *rows = r;
  return FPSCAN_OK;
}

int cuda_result(cudaError_t e, const char* what) {
  if (e != cudaSuccess)
    return fail(FPSCAN_ERR_CUDA, "%s: CUDA error %d (%s)", what, (int)e, cudaGetErrorString(e));
  return ok();
}

// Vectors per thread per chunk (NV).  FPSCAN_B200_NV=1 / 2 / 4 (4: fp32 only,
// other types use 2) overrides the choice below (a tuning knob read once per
// process).  Measured on B200 with dynamic row-unit scheduling, L2 flushed
// between calls:
//   forward: 2 -- the per-chunk block scan and barrier are amortised over
//     twice the data (bf16 8x2048x8192: 6342 vs 5839 GB/s with 1; fp32
//     4x8192x8192: 6849 vs 6306; fp16 16x5120x2048: 6392 vs 5992); launches
//     of at most 2^18 elements take 1 (fp32 2x256x512: 3.5 vs 5.0 us);
//   backward: 16-bit types 1 (bf16 8x2048x8192: 6404 vs 6179 GB/s; fp16
//     16x5120x2048: 6572 vs 6379); fp32 2 once rows exceed four per SM
//     (4x8192x8192: 6845 vs 6755), else 1 (2x256x65536: 5086 vs 4130).
int tuned_nv(bool forward, int dtype, int64_t rows, int64_t seqlen) {
  static const int env = [] {
    const char* v = getenv("FPSCAN_B200_NV");
    if (v && v[0] == '1') return 1;
    if (v && v[0] == '2') return 2;
    if (v && v[0] == '4') return 4;
    return 0;
  }();
  if (env) return env;
  if (forward) return rows * seqlen <= (int64_t(1) << 18) ? 1 : 2;
  if (dtype != FPSCAN_F32) return 1;
  return rows > 4 * (int64_t)num_sms_current() ? 2 : 1;
}

// Gated kernels (activation fused), measured at BASELINE config 4 (bf16):
// two vectors per thread in both directions -- the forward does more work
// per element (6.84 TB/s vs 5.48 with one); the two-pass backward fits the
// 3-CTA register budget at two vectors (5.98 TB/s vs 5.40 with one).
int tuned_nv_act(bool forward, int dtype, int act, int64_t rows, int64_t seqlen) {
  if (act == kActNone || dtype == FPSCAN_F32 || getenv("FPSCAN_B200_NV"))
    return tuned_nv(forward, dtype, rows, seqlen);
  return 2;
}

constexpr int64_t kRefMinL = 32, kRefMaxL = 65536;  // csrc/full_scan/full_scan.cu:207-233
constexpr int64_t kShardMaxL = int64_t(1) << 24;

#define FPSCAN_TRY(expr)          \
  do {                            \
    int _rc = (expr);             \
    if (_rc != FPSCAN_OK) return _rc; \
  } while (0)

}  // namespace

bool link_claims() {
  static const bool on = [] {
    const char* v = getenv("FPSCAN_B200_LINK_CLAIM");
    return !(v && v[0] == '0');
  }();
  return on;
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = getenv("FPSCAN_B200_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

int set_error(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return code;
}

}  // namespace fpscan

using namespace fpscan;

extern "C" {

int fpscan_abi_version(void) { return FPSCAN_ABI_VERSION; }

const char* fpscan_last_error(void) { return t_last_error.c_str(); }

}  // extern "C"

static int scan_fwd_impl(const void* gates, const void* tokens, void* out, int64_t batch,
                         int64_t dim, int64_t seqlen, int dtype, int reverse, int act,
                         void* stream) {
  if (act < kActNone || act > kActExp)
    return fail(FPSCAN_ERR_INVALID, "unknown gate activation code %d", act);
  int64_t rows = 0;
  FPSCAN_TRY(check_dtype(dtype));
  FPSCAN_TRY(check_shape(batch, dim, seqlen, kRefMinL, kRefMaxL, &rows));
  if (rows == 0) return ok();
  FPSCAN_TRY(check_ptr(gates, "gates"));
  FPSCAN_TRY(check_ptr(tokens, "tokens"));
  FPSCAN_TRY(check_ptr(out, "out"));
  const uintptr_t bytes = (uintptr_t)(rows * seqlen * dtype_size(dtype));
  const Span so{"out", (uintptr_t)out, (uintptr_t)out + bytes};
  const Span sg{"gates", (uintptr_t)gates, (uintptr_t)gates + bytes};
  const Span st{"tokens", (uintptr_t)tokens, (uintptr_t)tokens + bytes};
  for (const Span* in : {&sg, &st})
    if (overlaps(so, *in) && so.lo != in->lo)
      return fail(FPSCAN_ERR_INVALID, "out partially overlaps %s", in->name);
  FwdArgs a{gates, tokens, out, nullptr, nullptr, nullptr, rows, seqlen, dtype,
            reverse ? 1 : 0, num_sms_current(), static_cast<cudaStream_t>(stream)};
  a.nv = tuned_nv_act(true, dtype, act, rows, seqlen);
  a.act = act;
  a.sched = sched_counter(a.stream);
  return cuda_result(launch_fwd(a), "fpscan_scan_fwd launch");
}

extern "C" {

int fpscan_scan_fwd(const void* gates, const void* tokens, void* out, int64_t batch, int64_t dim,
                    int64_t seqlen, int dtype, int reverse, void* stream) {
  return scan_fwd_impl(gates, tokens, out, batch, dim, seqlen, dtype, reverse, kActNone, stream);
}

int fpscan_scan_fwd_act(const void* z, const void* tokens, void* out, int64_t batch, int64_t dim,
                        int64_t seqlen, int dtype, int reverse, int activation, void* stream) {
  return scan_fwd_impl(z, tokens, out, batch, dim, seqlen, dtype, reverse, activation, stream);
}

int64_t fpscan_scan_fwd_workspace_bytes(int64_t batch, int64_t dim, int64_t seqlen, int dtype) {
  int64_t rows = 0;
  if (check_dtype(dtype) != FPSCAN_OK) return 0;
  if (check_shape(batch, dim, seqlen, kRefMinL, kRefMaxL, &rows) != FPSCAN_OK) return 0;
  const int p = split_segments(rows, seqlen, dtype, split_slots(dtype, num_sms_current()));
  return split_workspace_bytes(rows, p);
}

int fpscan_scan_fwd_ws(const void* gates, const void* tokens, void* out, int64_t batch,
                       int64_t dim, int64_t seqlen, int dtype, int reverse, void* workspace,
                       int64_t workspace_bytes, void* stream) {
  int64_t rows = 0;
  FPSCAN_TRY(check_dtype(dtype));
  FPSCAN_TRY(check_shape(batch, dim, seqlen, kRefMinL, kRefMaxL, &rows));
  if (rows == 0) return ok();
  const int p = split_segments(rows, seqlen, dtype, split_slots(dtype, num_sms_current()));
  if (p <= 1) return fpscan_scan_fwd(gates, tokens, out, batch, dim, seqlen, dtype, reverse, stream);
  FPSCAN_TRY(check_ptr(gates, "gates"));
  FPSCAN_TRY(check_ptr(tokens, "tokens"));
  FPSCAN_TRY(check_ptr(out, "out"));
  FPSCAN_TRY(check_ptr(workspace, "workspace"));
  const int64_t need = split_workspace_bytes(rows, p);
  if (workspace_bytes < need)
    return fail(FPSCAN_ERR_INVALID, "workspace too small: %lld bytes, need %lld",
                (long long)workspace_bytes, (long long)need);
  const uintptr_t bytes = (uintptr_t)(rows * seqlen * dtype_size(dtype));
  const Span so{"out", (uintptr_t)out, (uintptr_t)out + bytes};
  const Span sg{"gates", (uintptr_t)gates, (uintptr_t)gates + bytes};
  const Span st{"tokens", (uintptr_t)tokens, (uintptr_t)tokens + bytes};
  const Span sw{"workspace", (uintptr_t)workspace, (uintptr_t)workspace + (uintptr_t)need};
  for (const Span* in : {&sg, &st})
    if (overlaps(so, *in) && so.lo != in->lo)
      return fail(FPSCAN_ERR_INVALID, "out partially overlaps %s", in->name);
  for (const Span* in : {&sg, &st, &so})
    if (overlaps(sw, *in)) return fail(FPSCAN_ERR_INVALID, "workspace overlaps %s", in->name);
  SplitArgs a{gates, tokens, out, workspace, rows, seqlen, p, dtype, reverse ? 1 : 0,
              static_cast<cudaStream_t>(stream)};
  return cuda_result(launch_split(a), "fpscan_scan_fwd_ws launch");
}

}  // extern "C"

static int scan_bwd_impl(const void* gates, const void* y, const void* grad_out, void* dgates,
                         void* dtokens, int64_t batch, int64_t dim, int64_t seqlen, int dtype,
                         int act, void* stream) {
  if (act < kActNone || act > kActExp)
    return fail(FPSCAN_ERR_INVALID, "unknown gate activation code %d", act);
  int64_t rows = 0;
  FPSCAN_TRY(check_dtype(dtype));
  FPSCAN_TRY(check_shape(batch, dim, seqlen, kRefMinL, kRefMaxL, &rows));
  if (rows == 0) return ok();
  FPSCAN_TRY(check_ptr(gates, "gates"));
  FPSCAN_TRY(check_ptr(y, "y"));
  FPSCAN_TRY(check_ptr(grad_out, "grad_out"));
  FPSCAN_TRY(check_ptr(dgates, "dgates"));
  FPSCAN_TRY(check_ptr(dtokens, "dtokens"));
  const uintptr_t bytes = (uintptr_t)(rows * seqlen * dtype_size(dtype));
  const Span in[3] = {{"gates", (uintptr_t)gates, (uintptr_t)gates + bytes},
                      {"y", (uintptr_t)y, (uintptr_t)y + bytes},
                      {"grad_out", (uintptr_t)grad_out, (uintptr_t)grad_out + bytes}};
  const Span o[2] = {{"dgates", (uintptr_t)dgates, (uintptr_t)dgates + bytes},
                     {"dtokens", (uintptr_t)dtokens, (uintptr_t)dtokens + bytes}};
  if (overlaps(o[0], o[1])) return fail(FPSCAN_ERR_INVALID, "dgates overlaps dtokens");
  for (const Span& os : o)
    for (const Span& is : in)
      if (overlaps(os, is)) return fail(FPSCAN_ERR_INVALID, "%s overlaps %s", os.name, is.name);
  BwdArgs a{gates,   y,       grad_out, dgates, dtokens, nullptr, nullptr,
            nullptr, rows,    seqlen,   dtype,  num_sms_current(),
            static_cast<cudaStream_t>(stream)};
  a.nv = tuned_nv_act(false, dtype, act, rows, seqlen);
  a.act = act;
  a.sched = sched_counter(a.stream);
  return cuda_result(launch_bwd(a), "fpscan_scan_bwd launch");
}

extern "C" {

int fpscan_scan_bwd(const void* gates, const void* y, const void* grad_out, void* dgates,
                    void* dtokens, int64_t batch, int64_t dim, int64_t seqlen, int dtype,
                    void* stream) {
  return scan_bwd_impl(gates, y, grad_out, dgates, dtokens, batch, dim, seqlen, dtype, kActNone,
                       stream);
}

int64_t fpscan_scan_bwd_workspace_bytes(int64_t batch, int64_t dim, int64_t seqlen, int dtype) {
  int64_t rows = 0;
  if (check_dtype(dtype) != FPSCAN_OK) return 0;
  if (check_shape(batch, dim, seqlen, kRefMinL, kRefMaxL, &rows) != FPSCAN_OK) return 0;
  const int p = split_bwd_segments(rows, seqlen, dtype, num_sms_current());
  return split_workspace_bytes(rows, p);
}

int fpscan_scan_bwd_ws(const void* gates, const void* y, const void* grad_out, void* dgates,
                       void* dtokens, int64_t batch, int64_t dim, int64_t seqlen, int dtype,
                       void* workspace, int64_t workspace_bytes, void* stream) {
  int64_t rows = 0;
  FPSCAN_TRY(check_dtype(dtype));
  FPSCAN_TRY(check_shape(batch, dim, seqlen, kRefMinL, kRefMaxL, &rows));
  if (rows == 0) return ok();
  const int p = split_bwd_segments(rows, seqlen, dtype, num_sms_current());
  if (p <= 1)
    return fpscan_scan_bwd(gates, y, grad_out, dgates, dtokens, batch, dim, seqlen, dtype, stream);
  FPSCAN_TRY(check_ptr(gates, "gates"));
  FPSCAN_TRY(check_ptr(y, "y"));
  FPSCAN_TRY(check_ptr(grad_out, "grad_out"));
  FPSCAN_TRY(check_ptr(dgates, "dgates"));
  FPSCAN_TRY(check_ptr(dtokens, "dtokens"));
  FPSCAN_TRY(check_ptr(workspace, "workspace"));
  const int64_t need = split_workspace_bytes(rows, p);
  if (workspace_bytes < need)
    return fail(FPSCAN_ERR_INVALID, "workspace too small: %lld bytes, need %lld",
                (long long)workspace_bytes, (long long)need);
  const uintptr_t bytes = (uintptr_t)(rows * seqlen * dtype_size(dtype));
  const Span all[6] = {{"gates", (uintptr_t)gates, (uintptr_t)gates + bytes},
                       {"y", (uintptr_t)y, (uintptr_t)y + bytes},
                       {"grad_out", (uintptr_t)grad_out, (uintptr_t)grad_out + bytes},
                       {"workspace", (uintptr_t)workspace, (uintptr_t)workspace + (uintptr_t)need},
                       {"dgates", (uintptr_t)dgates, (uintptr_t)dgates + bytes},
                       {"dtokens", (uintptr_t)dtokens, (uintptr_t)dtokens + bytes}};
  for (int i = 3; i < 6; ++i)
    for (int j = 0; j < i; ++j)
      if (overlaps(all[i], all[j]))
        return fail(FPSCAN_ERR_INVALID, "%s overlaps %s", all[i].name, all[j].name);
  SplitBwdArgs a{gates,  y,    grad_out, dgates, dtokens, workspace,
                 rows,   seqlen, p,      dtype,  static_cast<cudaStream_t>(stream)};
  return cuda_result(launch_split_bwd(a), "fpscan_scan_bwd_ws launch");
}

int fpscan_scan_bwd_act(const void* z, const void* y, const void* grad_out, void* dz,
                        void* dtokens, int64_t batch, int64_t dim, int64_t seqlen, int dtype,
                        int activation, void* stream) {
  return scan_bwd_impl(z, y, grad_out, dz, dtokens, batch, dim, seqlen, dtype, activation, stream);
}

int fpscan_scan_fwd_init(const void* gates, const void* tokens, void* out, const float* init,
                         int64_t batch, int64_t dim, int64_t seqlen, int dtype, int reverse,
                         void* stream) {
  int64_t rows = 0;
  FPSCAN_TRY(check_dtype(dtype));
  FPSCAN_TRY(check_shape(batch, dim, seqlen, kRefMinL, kRefMaxL, &rows));
  if (rows == 0) return ok();
  FPSCAN_TRY(check_ptr(gates, "gates"));
  FPSCAN_TRY(check_ptr(tokens, "tokens"));
  FPSCAN_TRY(check_ptr(out, "out"));
  if (!init) return fail(FPSCAN_ERR_INVALID, "init is NULL");
  const uintptr_t bytes = (uintptr_t)(rows * seqlen * dtype_size(dtype));
  const Span so{"out", (uintptr_t)out, (uintptr_t)out + bytes};
  const Span sg{"gates", (uintptr_t)gates, (uintptr_t)gates + bytes};
  const Span st{"tokens", (uintptr_t)tokens, (uintptr_t)tokens + bytes};
  for (const Span* in : {&sg, &st})
    if (overlaps(so, *in) && so.lo != in->lo)
      return fail(FPSCAN_ERR_INVALID, "out partially overlaps %s", in->name);
  FwdArgs a{gates, tokens, out, init, nullptr, nullptr, rows, seqlen, dtype, reverse ? 1 : 0,
            num_sms_current(), static_cast<cudaStream_t>(stream)};
  a.nv = tuned_nv(true, dtype, rows, seqlen);
  a.sched = sched_counter(a.stream);
  return cuda_result(launch_fwd(a), "fpscan_scan_fwd_init launch");
}

int fpscan_shard_fwd_reduce(const void* gates, const void* tokens, float* carry_a,
                            float* carry_b, int64_t rows, int64_t seqlen, int dtype,
                            void* stream) {
  int64_t r = 0;
  FPSCAN_TRY(check_dtype(dtype));
  FPSCAN_TRY(check_shape(rows, 1, seqlen, kRefMinL, kShardMaxL, &r));
  if (r == 0) return ok();
  FPSCAN_TRY(check_ptr(gates, "gates"));
  FPSCAN_TRY(check_ptr(tokens, "tokens"));
  if (!carry_a || !carry_b) return fail(FPSCAN_ERR_INVALID, "carry_a/carry_b is NULL");
  FwdArgs a{gates, tokens, nullptr, nullptr, carry_a, carry_b, r, seqlen, dtype, 0,
            num_sms_current(), static_cast<cudaStream_t>(stream)};
  a.nv = tuned_nv(true, dtype, r, seqlen);
  a.sched = sched_counter(a.stream);
  return cuda_result(launch_fwd(a), "fpscan_shard_fwd_reduce launch");
}

int fpscan_shard_fwd_scan(const void* gates, const void* tokens, void* out, const float* y_init,
                          int64_t rows, int64_t seqlen, int dtype, void* stream) {
  int64_t r = 0;
  FPSCAN_TRY(check_dtype(dtype));
  FPSCAN_TRY(check_shape(rows, 1, seqlen, kRefMinL, kShardMaxL, &r));
  if (r == 0) return ok();
  FPSCAN_TRY(check_ptr(gates, "gates"));
  FPSCAN_TRY(check_ptr(tokens, "tokens"));
  FPSCAN_TRY(check_ptr(out, "out"));
  if (!y_init) return fail(FPSCAN_ERR_INVALID, "y_init is NULL");
  FwdArgs a{gates, tokens, out, y_init, nullptr, nullptr, r, seqlen, dtype, 0,
            num_sms_current(), static_cast<cudaStream_t>(stream)};
  a.nv = tuned_nv(true, dtype, r, seqlen);
  a.sched = sched_counter(a.stream);
  return cuda_result(launch_fwd(a), "fpscan_shard_fwd_scan launch");
}

int fpscan_shard_bwd_reduce(const void* gates, const void* grad_out, float* carry_b,
                            int64_t rows, int64_t seqlen, int dtype, void* stream) {
  int64_t r = 0;
  FPSCAN_TRY(check_dtype(dtype));
  FPSCAN_TRY(check_shape(rows, 1, seqlen, kRefMinL, kShardMaxL, &r));
  if (r == 0) return ok();
  FPSCAN_TRY(check_ptr(gates, "gates"));
  FPSCAN_TRY(check_ptr(grad_out, "grad_out"));
  if (!carry_b) return fail(FPSCAN_ERR_INVALID, "carry_b is NULL");
  BwdArgs a{gates,   nullptr, grad_out, nullptr, nullptr, nullptr, nullptr,
            carry_b, r,       seqlen,   dtype,   num_sms_current(),
            static_cast<cudaStream_t>(stream)};
  a.nv = tuned_nv(false, dtype, r, seqlen);
  a.sched = sched_counter(a.stream);
  return cuda_result(launch_bwd(a), "fpscan_shard_bwd_reduce launch");
}

int fpscan_shard_bwd_scan(const void* gates, const void* y, const void* grad_out, void* dgates,
                          void* dtokens, const float* addend, const float* y_prev, int64_t rows,
                          int64_t seqlen, int dtype, void* stream) {
  int64_t r = 0;
  FPSCAN_TRY(check_dtype(dtype));
  FPSCAN_TRY(check_shape(rows, 1, seqlen, kRefMinL, kShardMaxL, &r));
  if (r == 0) return ok();
  FPSCAN_TRY(check_ptr(gates, "gates"));
  FPSCAN_TRY(check_ptr(y, "y"));
  FPSCAN_TRY(check_ptr(grad_out, "grad_out"));
  FPSCAN_TRY(check_ptr(dgates, "dgates"));
  FPSCAN_TRY(check_ptr(dtokens, "dtokens"));
  if (!addend || !y_prev) return fail(FPSCAN_ERR_INVALID, "addend/y_prev is NULL");
  BwdArgs a{gates,   y, grad_out, dgates, dtokens, addend, y_prev,
            nullptr, r, seqlen,   dtype,  num_sms_current(),
            static_cast<cudaStream_t>(stream)};
  a.nv = tuned_nv(false, dtype, r, seqlen);
  a.sched = sched_counter(a.stream);
  return cuda_result(launch_bwd(a), "fpscan_shard_bwd_scan launch");
}

int fpscan_carry_combine(const float* gathered, int world, int rank, int64_t rows, int reverse,
                         float* out, void* stream) {
  if (world < 1 || rank < 0 || rank >= world)
    return fail(FPSCAN_ERR_INVALID, "invalid world (%d) / rank (%d)", world, rank);
  if (rows < 0) return fail(FPSCAN_ERR_INVALID, "rows must be non-negative");
  if (rows == 0) return ok();
  if (!gathered || !out) return fail(FPSCAN_ERR_INVALID, "gathered/out is NULL");
  return cuda_result(launch_carry_combine(gathered, world, rank, rows, reverse ? 1 : 0, out,
                                          static_cast<cudaStream_t>(stream)),
                     "fpscan_carry_combine launch");
}

int fpscan_debug_bounds(void* stream) {
  bounds_probe_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>();
  if (cudaGetLastError() != cudaSuccess) return -1;
#ifdef FPSCAN_DEBUG_BOUNDS
  return 1;
#else
  return 0;
#endif
}

int fpscan_set_wait_limit_ns(uint64_t ns) {
  if (ns < 1000000ull || ns > 600000000000ull)
    return fail(FPSCAN_ERR_INVALID, "wait limit must be in [1 ms, 600 s] (got %llu ns)",
                (unsigned long long)ns);
  const unsigned long long v = ns;
  return cuda_result(cudaMemcpyToSymbol(g_wait_limit_ns, &v, sizeof(v)),
                     "fpscan_set_wait_limit_ns");
}

int fpscan_status_snapshot(unsigned* dst, void* stream) {
  if (!dst) return fail(FPSCAN_ERR_INVALID, "dst is NULL");
  status_take_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(dst);
  return cuda_result(cudaGetLastError(), "fpscan_status_snapshot launch");
}

int fpscan_device_status(unsigned* status, int clear) {
  if (!status) return fail(FPSCAN_ERR_INVALID, "status is NULL");
  unsigned v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_status, sizeof(v));
  if (e != cudaSuccess) return cuda_result(e, "fpscan_device_status read");
  if (clear && v) {
    const unsigned zero = 0;
    e = cudaMemcpyToSymbol(g_status, &zero, sizeof(zero));
    if (e != cudaSuccess) return cuda_result(e, "fpscan_device_status clear");
  }
  *status = v;
  return ok();
}

}  // extern "C"

extern "C" {

int fpscan_scan_fwd_anylen(const void* gates, const void* tokens, void* out, int64_t batch,
                           int64_t dim, int64_t seqlen, int dtype, int reverse, void* stream) {
  int64_t rows = 0;
  FPSCAN_TRY(check_dtype(dtype));
  FPSCAN_TRY(check_shape_any(batch, dim, seqlen, &rows));
  if (rows == 0) return ok();
  FPSCAN_TRY(check_ptr(gates, "gates"));
  FPSCAN_TRY(check_ptr(tokens, "tokens"));
  FPSCAN_TRY(check_ptr(out, "out"));
  const uintptr_t bytes = (uintptr_t)(rows * seqlen * dtype_size(dtype));
  const Span so{"out", (uintptr_t)out, (uintptr_t)out + bytes};
  const Span sg{"gates", (uintptr_t)gates, (uintptr_t)gates + bytes};
  const Span st{"tokens", (uintptr_t)tokens, (uintptr_t)tokens + bytes};
  for (const Span* in : {&sg, &st})
    if (overlaps(so, *in) && so.lo != in->lo)
      return fail(FPSCAN_ERR_INVALID, "out partially overlaps %s", in->name);
  AnyArgs a{};
  a.gates = gates;
  a.tokens = tokens;
  a.out = out;
  a.rows = rows;
  a.seqlen = seqlen;
  a.dtype = dtype;
  a.reverse = reverse ? 1 : 0;
  a.backward = 0;
  a.num_sms = num_sms_current();
  a.stream = static_cast<cudaStream_t>(stream);
  // measured on B200 (bf16 / fp32, (8, 2048, 8191) and (16, 5120, 16383)):
  // two vectors per thread, 5.3-5.7 TB/s bf16 vs 4.3 with one
  a.nv = 2;
  if (const char* v = getenv("FPSCAN_B200_ANY_FWD_NV")) a.nv = v[0] == '1' ? 1 : 2;
  return cuda_result(launch_anylen(a), "fpscan_scan_fwd_anylen launch");
}

int fpscan_scan_bwd_anylen(const void* gates, const void* y, const void* grad_out, void* dgates,
                           void* dtokens, int64_t batch, int64_t dim, int64_t seqlen, int dtype,
                           void* stream) {
  int64_t rows = 0;
  FPSCAN_TRY(check_dtype(dtype));
  FPSCAN_TRY(check_shape_any(batch, dim, seqlen, &rows));
  if (rows == 0) return ok();
  FPSCAN_TRY(check_ptr(gates, "gates"));
  FPSCAN_TRY(check_ptr(y, "y"));
  FPSCAN_TRY(check_ptr(grad_out, "grad_out"));
  FPSCAN_TRY(check_ptr(dgates, "dgates"));
  FPSCAN_TRY(check_ptr(dtokens, "dtokens"));
  const uintptr_t bytes = (uintptr_t)(rows * seqlen * dtype_size(dtype));
  const Span in[3] = {{"gates", (uintptr_t)gates, (uintptr_t)gates + bytes},
                      {"y", (uintptr_t)y, (uintptr_t)y + bytes},
                      {"grad_out", (uintptr_t)grad_out, (uintptr_t)grad_out + bytes}};
  const Span o[2] = {{"dgates", (uintptr_t)dgates, (uintptr_t)dgates + bytes},
                     {"dtokens", (uintptr_t)dtokens, (uintptr_t)dtokens + bytes}};
  if (overlaps(o[0], o[1])) return fail(FPSCAN_ERR_INVALID, "dgates overlaps dtokens");
  for (const Span& os : o)
    for (const Span& is : in)
      if (overlaps(os, is)) return fail(FPSCAN_ERR_INVALID, "%s overlaps %s", os.name, is.name);
  AnyArgs a{};
  a.gates = gates;
  a.y = y;
  a.grad_out = grad_out;
  a.dgates = dgates;
  a.dtokens = dtokens;
  a.rows = rows;
  a.seqlen = seqlen;
  a.dtype = dtype;
  a.backward = 1;
  a.num_sms = num_sms_current();
  a.stream = static_cast<cudaStream_t>(stream);
  // two vectors per thread (fp32 6.3 TB/s vs 5.3; bf16, at a 2-CTA register
  // budget, 5.2-5.6 vs 5.0 with one)
  a.nv = 2;
  if (const char* v = getenv("FPSCAN_B200_ANY_BWD_NV")) a.nv = v[0] == '2' ? 2 : 1;
  return cuda_result(launch_anylen(a), "fpscan_scan_bwd_anylen launch");
}

}  // extern "C"

// ------------------------------------------------------------------ channel-last
static int check_cl(int64_t batch, int64_t seqlen, int64_t dim, int dtype) {
  FPSCAN_TRY(check_dtype(dtype));
  if (batch < 0 || dim < 0 || seqlen < 1)
    return fail(FPSCAN_ERR_INVALID,
                "batch (%lld) and dim (%lld) must be non-negative and seqlen (%lld) >= 1",
                (long long)batch, (long long)dim, (long long)seqlen);
  if ((dim * dtype_size(dtype)) % 16 != 0)
    return fail(FPSCAN_ERR_INVALID,
                "dim (%lld) must be a multiple of %d for this dtype (16-byte rows)", (long long)dim,
                16 / dtype_size(dtype));
  if (batch >= (int64_t(1) << 31) || seqlen >= (int64_t(1) << 31) - 64 ||
      dim >= (int64_t(1) << 31))
    return fail(FPSCAN_ERR_INVALID, "batch, seqlen and dim must each be below 2^31");
  if (batch != 0 && dim != 0 && batch * seqlen > INT64_MAX / dim / 8)
    return fail(FPSCAN_ERR_INVALID, "tensor too large");
  return FPSCAN_OK;
}

extern "C" {

int64_t fpscan_cl_workspace_bytes(int64_t batch, int64_t seqlen, int64_t dim, int dtype,
                                  int backward) {
  if (check_cl(batch, seqlen, dim, dtype) != FPSCAN_OK) return 0;
  return cl_workspace_bytes(batch, seqlen, dim, dtype, backward != 0);
}

int fpscan_scan_fwd_cl(const void* gates, const void* tokens, void* out, int64_t batch,
                       int64_t seqlen, int64_t dim, int dtype, int reverse, void* workspace,
                       int64_t workspace_bytes, void* stream) {
  FPSCAN_TRY(check_cl(batch, seqlen, dim, dtype));
  if (batch == 0 || dim == 0) return ok();
  FPSCAN_TRY(check_ptr(gates, "gates"));
  FPSCAN_TRY(check_ptr(tokens, "tokens"));
  FPSCAN_TRY(check_ptr(out, "out"));
  FPSCAN_TRY(check_ptr(workspace, "workspace"));
  const int64_t need = cl_workspace_bytes(batch, seqlen, dim, dtype, false);
  if (workspace_bytes < need)
    return fail(FPSCAN_ERR_INVALID, "workspace too small: %lld bytes, need %lld",
                (long long)workspace_bytes, (long long)need);
  const uintptr_t bytes = (uintptr_t)(batch * seqlen * dim * dtype_size(dtype));
  const Span so{"out", (uintptr_t)out, (uintptr_t)out + bytes};
  const Span sg{"gates", (uintptr_t)gates, (uintptr_t)gates + bytes};
  const Span st{"tokens", (uintptr_t)tokens, (uintptr_t)tokens + bytes};
  const Span sw{"workspace", (uintptr_t)workspace, (uintptr_t)workspace + (uintptr_t)need};
  for (const Span* in : {&sg, &st})
    if (overlaps(so, *in) && so.lo != in->lo)
      return fail(FPSCAN_ERR_INVALID, "out partially overlaps %s", in->name);
  for (const Span* t : {&so, &sg, &st})
    if (overlaps(sw, *t)) return fail(FPSCAN_ERR_INVALID, "workspace overlaps %s", t->name);
  ClArgs a{};
  a.gates = gates;
  a.tokens = tokens;
  a.out = out;
  a.workspace = workspace;
  a.workspace_bytes = (uint64_t)workspace_bytes;
  a.batch = batch;
  a.seqlen = seqlen;
  a.dim = dim;
  a.dtype = dtype;
  a.reverse = reverse ? 1 : 0;
  a.backward = 0;
  a.stream = static_cast<cudaStream_t>(stream);
  return cuda_result(launch_cl(a), "fpscan_scan_fwd_cl launch");
}

int fpscan_scan_bwd_cl(const void* gates, const void* y, const void* grad_out, void* dgates,
                       void* dtokens, int64_t batch, int64_t seqlen, int64_t dim, int dtype,
                       void* workspace, int64_t workspace_bytes, void* stream) {
  FPSCAN_TRY(check_cl(batch, seqlen, dim, dtype));
  if (batch == 0 || dim == 0) return ok();
  FPSCAN_TRY(check_ptr(gates, "gates"));
  FPSCAN_TRY(check_ptr(y, "y"));
  FPSCAN_TRY(check_ptr(grad_out, "grad_out"));
  FPSCAN_TRY(check_ptr(dgates, "dgates"));
  FPSCAN_TRY(check_ptr(dtokens, "dtokens"));
  FPSCAN_TRY(check_ptr(workspace, "workspace"));
  const int64_t need = cl_workspace_bytes(batch, seqlen, dim, dtype, true);
  if (workspace_bytes < need)
    return fail(FPSCAN_ERR_INVALID, "workspace too small: %lld bytes, need %lld",
                (long long)workspace_bytes, (long long)need);
  const uintptr_t bytes = (uintptr_t)(batch * seqlen * dim * dtype_size(dtype));
  const Span all[6] = {{"gates", (uintptr_t)gates, (uintptr_t)gates + bytes},
                       {"y", (uintptr_t)y, (uintptr_t)y + bytes},
                       {"grad_out", (uintptr_t)grad_out, (uintptr_t)grad_out + bytes},
                       {"workspace", (uintptr_t)workspace, (uintptr_t)workspace + (uintptr_t)need},
                       {"dgates", (uintptr_t)dgates, (uintptr_t)dgates + bytes},
                       {"dtokens", (uintptr_t)dtokens, (uintptr_t)dtokens + bytes}};
  for (int i = 3; i < 6; ++i)
    for (int j = 0; j < i; ++j)
      if (overlaps(all[i], all[j]))
        return fail(FPSCAN_ERR_INVALID, "%s overlaps %s", all[i].name, all[j].name);
  ClArgs a{};
  a.gates = gates;
  a.y = y;
  a.grad_out = grad_out;
  a.dgates = dgates;
  a.dtokens = dtokens;
  a.workspace = workspace;
  a.workspace_bytes = (uint64_t)workspace_bytes;
  a.batch = batch;
  a.seqlen = seqlen;
  a.dim = dim;
  a.dtype = dtype;
  a.backward = 1;
  a.stream = static_cast<cudaStream_t>(stream);
  return cuda_result(launch_cl(a), "fpscan_scan_bwd_cl launch");
}

}  // extern "C"

// ------------------------------------------------------------------ rank links
// Mailbox of one rank (cudaMalloc'd once per (rows, depth); 256-byte aligned
// regions):
//   fwd[depth][rows]  64-bit words (epoch << 32 | value) from rank r-1
//   bwd[depth][rows]  64-bit words from rank r+1
//   fwd_ack[rows]     u32: epochs of forward words rank r+1 has taken
//   bwd_ack[rows]     u32: epochs of backward words rank r-1 has taken
//   zeros[rows]       fp32, never written
// A call with epoch e uses ring slot e % depth; epochs start at 1 and are
// counted per direction, so a producer waits for ack >= e - depth.
namespace {
struct MailboxLayout {
  int64_t fwd, bwd, fwd_ack, bwd_ack, zeros, total;
};
MailboxLayout mailbox_layout(int64_t rows, int depth) {
  auto up = [](int64_t b) { return (b + 255) / 256 * 256; };
  const int64_t ring = up((int64_t)depth * rows * 8), one = up(rows * 4);
  MailboxLayout m;
  m.fwd = 0;
  m.bwd = m.fwd + ring;
  m.fwd_ack = m.bwd + ring;
  m.bwd_ack = m.fwd_ack + one;
  m.zeros = m.bwd_ack + one;
  m.total = m.zeros + one;
  return m;
}
template <typename P>
P* at(void* base, int64_t off) {
  return reinterpret_cast<P*>(static_cast<char*>(base) + off);
}
int check_link(int64_t rows, int depth) {
  if (rows <= 0 || rows > (int64_t(1) << 31))
    return fail(FPSCAN_ERR_INVALID, "link rows must be in [1, 2^31] (got %lld)", (long long)rows);
  if (depth < 1 || depth > 64)
    return fail(FPSCAN_ERR_INVALID, "link depth must be in [1, 64] (got %d)", depth);
  return FPSCAN_OK;
}
}  // namespace

extern "C" {

int64_t fpscan_link_bytes(int64_t rows, int depth) {
  if (check_link(rows, depth) != FPSCAN_OK) return 0;
  return mailbox_layout(rows, depth).total;
}

int fpscan_link_create(int64_t rows, int depth, void** mailbox) {
  FPSCAN_TRY(check_link(rows, depth));
  if (mailbox == nullptr) return fail(FPSCAN_ERR_INVALID, "mailbox is NULL");
  const int64_t bytes = mailbox_layout(rows, depth).total;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, (size_t)bytes);
  if (e == cudaSuccess) e = cudaMemset(p, 0, (size_t)bytes);
  if (e != cudaSuccess) {
    if (p) cudaFree(p);
    return cuda_result(e, "fpscan_link_create");
  }
  *mailbox = p;
  return ok();
}

int fpscan_link_destroy(void* mailbox) {
  if (mailbox == nullptr) return ok();
  return cuda_result(cudaFree(mailbox), "fpscan_link_destroy");
}

int fpscan_link_ipc_handle(void* mailbox, void* handle) {
  if (mailbox == nullptr || handle == nullptr)
    return fail(FPSCAN_ERR_INVALID, "mailbox and handle must not be NULL");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, mailbox);
  if (e != cudaSuccess) return cuda_result(e, "fpscan_link_ipc_handle");
  memcpy(handle, &h, sizeof(h));
  return ok();
}

int fpscan_link_open(const void* handle, void** peer_mailbox) {
  if (handle == nullptr || peer_mailbox == nullptr)
    return fail(FPSCAN_ERR_INVALID, "handle and peer_mailbox must not be NULL");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_result(e, "fpscan_link_open");
  *peer_mailbox = p;
  return ok();
}

int fpscan_link_close(void* peer_mailbox) {
  if (peer_mailbox == nullptr) return ok();
  return cuda_result(cudaIpcCloseMemHandle(peer_mailbox), "fpscan_link_close");
}

int fpscan_shard_fwd_link(const void* gates, const void* tokens, void* out, float* init_record,
                          int64_t rows, int64_t seqlen, int dtype, void* local, void* prev,
                          void* next, uint32_t epoch, int depth, void* stream) {
  FPSCAN_TRY(check_dtype(dtype));
  FPSCAN_TRY(check_link(rows, depth));
  if (local == nullptr) return fail(FPSCAN_ERR_INVALID, "local mailbox is NULL");
  if (prev == nullptr && next == nullptr)
    return fail(FPSCAN_ERR_INVALID, "a linked scan needs an upstream or a downstream rank");
  if (epoch == 0) return fail(FPSCAN_ERR_INVALID, "epoch 0 is reserved");
  // Two vectors per thread where a row spans more than one such chunk:
  // measured at config 5 with claimed row units, 2 / 4 GPUs: 12834 / 24973
  // GB/s against 11615 / 21692 with one.  FPSCAN_B200_LINK_FWD_NV=1 forces
  // one.
  static const bool nv_one = [] {
    const char* v = getenv("FPSCAN_B200_LINK_FWD_NV");
    return v && v[0] == '1';
  }();
  const int64_t chunk = (int64_t)kThreads * (16 / dtype_size(dtype));
  const int nv = (!nv_one && seqlen > 2 * chunk) ? 2 : 1;
  if (!is_pow2(seqlen) || seqlen <= chunk || seqlen > kShardMaxL)
    return fail(FPSCAN_ERR_INVALID,
                "linked scan: local seqlen must be a power of 2 > %lld and <= %lld (got %lld)",
                (long long)chunk, (long long)kShardMaxL, (long long)seqlen);
  FPSCAN_TRY(check_ptr(gates, "gates"));
  FPSCAN_TRY(check_ptr(tokens, "tokens"));
  FPSCAN_TRY(check_ptr(out, "out"));
  const MailboxLayout m = mailbox_layout(rows, depth);
  const int64_t slot = (int64_t)(epoch % (uint32_t)depth) * rows;
  FwdArgs a{gates, tokens, out, nullptr, nullptr, nullptr, rows, seqlen, dtype, 0,
            num_sms_current(), static_cast<cudaStream_t>(stream)};
  a.nv = nv;
  a.link = (prev ? 1 : 0) | (next ? 2 : 0);
  a.lk.epoch = epoch;
  a.lk.depth = (uint32_t)depth;
  if (prev) {
    a.lk.in_word = at<uint64_t>(local, m.fwd) + slot;
    a.lk.ack_out = at<uint32_t>(prev, m.fwd_ack);
    a.lk.in_record = init_record;
  }
  if (next) {
    a.lk.out_word = at<uint64_t>(next, m.fwd) + slot;
    a.lk.ack_in = at<uint32_t>(local, m.fwd_ack);
  }
  a.sched = link_claims() ? sched_counter(a.stream) : nullptr;
  return cuda_result(launch_fwd(a), "fpscan_shard_fwd_link launch");
}

int fpscan_shard_bwd_link(const void* gates, const void* y, const void* grad_out, void* dgates,
                          void* dtokens, const float* y_prev, int64_t rows, int64_t seqlen,
                          int dtype, void* local, void* prev, void* next, uint32_t epoch,
                          int depth, void* stream) {
  FPSCAN_TRY(check_dtype(dtype));
  FPSCAN_TRY(check_link(rows, depth));
  if (local == nullptr) return fail(FPSCAN_ERR_INVALID, "local mailbox is NULL");
  if (prev == nullptr && next == nullptr)
    return fail(FPSCAN_ERR_INVALID, "a linked scan needs an upstream or a downstream rank");
  if (epoch == 0) return fail(FPSCAN_ERR_INVALID, "epoch 0 is reserved");
  if (prev != nullptr && y_prev == nullptr)
    return fail(FPSCAN_ERR_INVALID, "y_prev is required on every rank but the first");
  const int nv = 2;
  const int64_t chunk = (int64_t)kThreads * (16 / dtype_size(dtype)) * nv;
  if (!is_pow2(seqlen) || seqlen <= chunk || seqlen > kShardMaxL)
    return fail(FPSCAN_ERR_INVALID,
                "linked backward: local seqlen must be a power of 2 > %lld and <= %lld (got %lld)",
                (long long)chunk, (long long)kShardMaxL, (long long)seqlen);
  FPSCAN_TRY(check_ptr(gates, "gates"));
  FPSCAN_TRY(check_ptr(y, "y"));
  FPSCAN_TRY(check_ptr(grad_out, "grad_out"));
  FPSCAN_TRY(check_ptr(dgates, "dgates"));
  FPSCAN_TRY(check_ptr(dtokens, "dtokens"));
  const MailboxLayout m = mailbox_layout(rows, depth);
  const int64_t slot = (int64_t)(epoch % (uint32_t)depth) * rows;
  BwdArgs a{gates,   y,       grad_out, dgates, dtokens, nullptr, nullptr,
            nullptr, rows,    seqlen,   dtype,  num_sms_current(),
            static_cast<cudaStream_t>(stream)};
  a.nv = nv;
  a.y_prev = y_prev ? y_prev : at<float>(local, m.zeros);
  a.link = (next ? 1 : 0) | (prev ? 2 : 0);
  a.lk.epoch = epoch;
  a.lk.depth = (uint32_t)depth;
  if (next) {
    a.lk.in_word = at<uint64_t>(local, m.bwd) + slot;
    a.lk.ack_out = at<uint32_t>(next, m.bwd_ack);
  }
  if (prev) {
    a.lk.out_word = at<uint64_t>(prev, m.bwd) + slot;
    a.lk.ack_in = at<uint32_t>(local, m.bwd_ack);
  }
  a.sched = link_claims() ? sched_counter(a.stream) : nullptr;
  return cuda_result(launch_bwd(a), "fpscan_shard_bwd_link launch");
}

}  // extern "C"
