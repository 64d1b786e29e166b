// fpscan_scan_fwd_noalloc: the forward / reverse scan for callers that cannot
// allocate device memory.
//
// Some callers of this library are not allowed to allocate GPU memory once
// they are running: a host application that hands the library a fixed memory
// budget and owns every allocation, a latency-critical service that forbids
// cudaMalloc/cudaFree after start-up because both can synchronise the whole
// device, or C code without a caching allocator that would otherwise have to
// cudaMalloc a workspace on every call.  fpscan_scan_fwd_ws needs a caller
// workspace for few-channel, long-sequence shapes (rows split across CTAs);
// this entry point instead uses a fixed scratch array that lives in the
// library's own device memory.
//
// The scratch is a file-scope __device__ array of kNoAllocScratchBytes
// (enough for kNoAllocMaxSegments split segments); every GPU that loads the
// library holds it until the process exits.  Its host-side name is only a
// stand-in, so the device address is looked up with cudaGetSymbolAddress,
// once per device, with that device current, by the first call on that
// device.  That set-up enqueues no GPU work (a __device__ array starts at
// zero when the module loads), but make the first call on each device before
// any stream capture all the same.  All calls share the array and it keeps
// the last call's contents: the tile counter is cleared by every call (an
// async memset on the call's own stream, ordered before its kernel) and the
// status words carry a per-call epoch, so nothing else must start at zero;
// calls that overlap on the GPU (two streams, or two host threads) race on
// it and must not be issued.
#include "../../include/fpscan_b200.h"
#include "common.cuh"
#include "internal.h"

#include <mutex>

namespace fpscan {
namespace {

constexpr int64_t kNoAllocMaxSegments = 512;
constexpr int64_t kNoAllocScratchBytes = 256 + 16 * kNoAllocMaxSegments;  // 8,448 bytes

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_setup_mutex;
void* g_scratch_addr[64] = {nullptr};

// Device address of the scratch array on the current device (set up once).
cudaError_t scratch_for_current_device(void** addr) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_addr[dev] = p;
  }
  *addr = g_scratch_addr[dev];
  return cudaSuccess;
}

}  // namespace
}  // namespace fpscan

using namespace fpscan;

extern "C" int fpscan_scan_fwd_noalloc(const void* gates, const void* tokens, void* out,
                                       int64_t batch, int64_t dim, int64_t seqlen, int dtype,
                                       int reverse, void* stream) {
  const int64_t need = fpscan_scan_fwd_workspace_bytes(batch, dim, seqlen, dtype);
  if (need > kNoAllocScratchBytes)
    return set_error(FPSCAN_ERR_INVALID,
                     "fpscan_scan_fwd_noalloc: this shape needs %lld bytes of scratch, above the "
                     "fixed %lld (%lld split segments); use fpscan_scan_fwd_ws",
                     (long long)need, (long long)kNoAllocScratchBytes,
                     (long long)kNoAllocMaxSegments);
  if (need == 0)  // no scratch needed: the one-CTA-per-row kernel
    return fpscan_scan_fwd(gates, tokens, out, batch, dim, seqlen, dtype, reverse, stream);
  void* scratch = nullptr;
  const cudaError_t e = scratch_for_current_device(&scratch);
  if (e != cudaSuccess)
    return set_error(FPSCAN_ERR_CUDA, "fpscan_scan_fwd_noalloc set-up: CUDA error %d (%s)",
                     (int)e, cudaGetErrorString(e));
  return fpscan_scan_fwd_ws(gates, tokens, out, batch, dim, seqlen, dtype, reverse, scratch,
                            kNoAllocScratchBytes, stream);
}
