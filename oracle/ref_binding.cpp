// ORACLE — test infrastructure only.  Binds the reference's own host
// launcher warpscan_fwd (csrc/full_scan/full_scan.h:26-36, defined there and
// in csrc/full_scan/full_scan.cu) under the reference's Python name
// fullscan_forward (csrc/main.cpp:10), so tests can run the reference kernel,
// compiled from its unmodified sources, next to fpscan_b200 on a B200.
// The reference's experimental dimwise kernels are not built.
#include <torch/extension.h>

#include "full_scan/full_scan.h"

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("fullscan_forward", &warpscan_fwd, "reference full scan forward (CUDA)");
}
