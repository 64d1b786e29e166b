// Thin torch binding over the C ABI (include/fpscan_b200.h): the fast path of
// fpscan_b200.ops for the reference's own entry points.  It plays the role of
// the reference's pybind module (csrc/main.cpp:10, fullscan_forward) -- tensor
// checks, output allocation, the caller's current stream -- in C++, so a
// call costs what the reference's does instead of a Python + ctypes round
// trip.  All work is done by libfpscan_b200.so; this file has no kernels.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <map>
#include <mutex>
#include <tuple>

#include "../../include/fpscan_b200.h"

namespace {

int dtype_code(const at::Tensor& t) {
  switch (t.scalar_type()) {
    case at::kFloat:
      return FPSCAN_F32;
    case at::kHalf:
      return FPSCAN_F16;
    case at::kBFloat16:
      return FPSCAN_BF16;
    default:
      TORCH_CHECK(false, "tokens must be float16 or bfloat16 or float32");
  }
  return -1;
}

// Same conditions and order as ops.validate (CHECK_INPUT of
// csrc/full_scan/full_scan.h:7-15, then shapes); the C ABI re-checks sizes,
// alignment and overlap.
void check_pair(const at::Tensor& gates, const at::Tensor& tokens, const char* gname) {
  TORCH_CHECK(gates.is_cuda(), gname, " must be a CUDA tensor");
  TORCH_CHECK(tokens.is_cuda(), "tokens must be a CUDA tensor");
  TORCH_CHECK(gates.is_contiguous(), gname, " must be contiguous");
  TORCH_CHECK(tokens.is_contiguous(), "tokens must be contiguous");
  TORCH_CHECK(tokens.dim() == 3, "tokens must be 3-D (batch, dim, seqlen)");
  TORCH_CHECK(gates.sizes() == tokens.sizes(), gname, " and tokens must have the same shape");
  TORCH_CHECK(gates.scalar_type() == tokens.scalar_type(), gname,
              " dtype must equal tokens dtype");
  TORCH_CHECK(gates.device() == tokens.device(), gname, " and tokens must be on the same device");
}

// Workspaces of the split-row paths, one per (device, stream, kind), zeroed
// once when (re)allocated; calls on one stream are ordered, so they may
// share it.  Kept for the life of the process (a few KB each).
at::Tensor workspace(const at::Tensor& like, int64_t bytes, int kind) {
  static std::mutex mu;
  static std::map<std::tuple<int, void*, int>, at::Tensor> cache;
  const auto key = std::make_tuple((int)like.get_device(),
                                   (void*)at::cuda::getCurrentCUDAStream().stream(), kind);
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it != cache.end() && it->second.numel() >= bytes) return it->second;
  at::Tensor w = at::zeros({std::max<int64_t>(bytes, 1 << 16)}, like.options().dtype(at::kByte));
  cache[key] = w;
  return w;
}

void raise_on(int rc, const char* what) {
  if (rc != FPSCAN_OK) TORCH_CHECK(false, what, ": ", fpscan_last_error());
}

at::Tensor fullscan_forward(const at::Tensor& gates, const at::Tensor& tokens, at::Tensor out,
                            bool reverse) {
  check_pair(gates, tokens, "gates");
  TORCH_CHECK(out.sizes() == tokens.sizes() && out.scalar_type() == tokens.scalar_type() &&
                  out.device() == tokens.device(),
              "out must match tokens in shape, dtype and device");
  TORCH_CHECK(out.is_contiguous(), "out must be contiguous");
  const int code = dtype_code(tokens);
  const int64_t b = tokens.size(0), d = tokens.size(1), l = tokens.size(2);
  const c10::cuda::CUDAGuard guard(tokens.device());
  void* stream = at::cuda::getCurrentCUDAStream().stream();
  const int64_t ws = fpscan_scan_fwd_workspace_bytes(b, d, l, code);
  if (ws > 0) {
    // few, long rows: the split-row kernel and its workspace
    at::Tensor w = workspace(tokens, ws, 0);
    raise_on(fpscan_scan_fwd_ws(gates.data_ptr(), tokens.data_ptr(), out.data_ptr(), b, d, l, code,
                                reverse ? 1 : 0, w.data_ptr(), w.numel(), stream),
             "fpscan_scan_fwd_ws");
  } else {
    raise_on(fpscan_scan_fwd(gates.data_ptr(), tokens.data_ptr(), out.data_ptr(), b, d, l, code,
                             reverse ? 1 : 0, stream),
             "fpscan_scan_fwd");
  }
  return out;
}

at::Tensor scan_forward(const at::Tensor& gates, const at::Tensor& tokens, bool reverse) {
  return fullscan_forward(gates, tokens, at::empty_like(tokens), reverse);
}

std::tuple<at::Tensor, at::Tensor> scan_backward(const at::Tensor& gates, const at::Tensor& y,
                                                 const at::Tensor& grad_out) {
  check_pair(gates, grad_out, "gates");
  check_pair(y, grad_out, "y");
  const int code = dtype_code(grad_out);
  const int64_t b = grad_out.size(0), d = grad_out.size(1), l = grad_out.size(2);
  const c10::cuda::CUDAGuard guard(grad_out.device());
  at::Tensor dgates = at::empty_like(grad_out), dtokens = at::empty_like(grad_out);
  void* stream = at::cuda::getCurrentCUDAStream().stream();
  const int64_t ws = fpscan_scan_bwd_workspace_bytes(b, d, l, code);
  if (ws > 0) {
    // few, long rows: the split-row backward and its workspace
    at::Tensor w = workspace(grad_out, ws, 1);
    raise_on(fpscan_scan_bwd_ws(gates.data_ptr(), y.data_ptr(), grad_out.data_ptr(),
                                dgates.data_ptr(), dtokens.data_ptr(), b, d, l, code,
                                w.data_ptr(), w.numel(), stream),
             "fpscan_scan_bwd_ws");
  } else {
    raise_on(fpscan_scan_bwd(gates.data_ptr(), y.data_ptr(), grad_out.data_ptr(),
                             dgates.data_ptr(), dtokens.data_ptr(), b, d, l, code, stream),
             "fpscan_scan_bwd");
  }
  return {dgates, dtokens};
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("fullscan_forward", &fullscan_forward,
        "fullscan_forward(gates, tokens, out, reverse) -> out (the reference extension's contract)");
  m.def("scan_forward", &scan_forward, "scan_forward(gates, tokens, reverse) -> out");
  m.def("scan_backward", &scan_backward,
        "scan_backward(gates, y, grad_out) -> (dgates, dtokens), the fused PScan backward");
  m.def("abi_version", []() { return fpscan_abi_version(); });
}
