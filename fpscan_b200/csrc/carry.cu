// Carry combination for the sequence-sharded mode (no reference counterpart:
// the reference has no multi-GPU path).
//
// After an all-gather every rank holds, for each shard q and row, the affine
// map (A_q, B_q) of that shard: y_out = A_q * y_in + B_q.  Forward: rank r's
// initial state is the composition of shards 0..r-1 applied to 0.  Backward
// (reverse): the value entering rank r from the right is the composition of
// shards world-1..r+1.  The first shard in the fold contributes B directly so
// that a non-finite A never meets the zero start state.
#include "common.cuh"
#include "internal.h"

namespace fpscan {

__global__ void carry_combine_kernel(const float* __restrict__ gathered, int world, int rank,
                                     int64_t rows, int reverse, float* __restrict__ out) {
  const int64_t row = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= rows) return;
  float v = 0.f;
  bool first = true;
  if (!reverse) {
    for (int q = 0; q < rank; ++q) {
      const float A = gathered[((int64_t)q * 2 + 0) * rows + row];
      const float B = gathered[((int64_t)q * 2 + 1) * rows + row];
      v = first ? B : fmaf(A, v, B);
      first = false;
    }
  } else {
    for (int q = world - 1; q > rank; --q) {
      const float A = gathered[((int64_t)q * 2 + 0) * rows + row];
      const float B = gathered[((int64_t)q * 2 + 1) * rows + row];
      v = first ? B : fmaf(A, v, B);
      first = false;
    }
  }
  out[row] = v;
}

cudaError_t launch_carry_combine(const float* gathered, int world, int rank, int64_t rows,
                                 int reverse, float* out, cudaStream_t stream) {
  const int threads = 256;
  const int64_t blocks = (rows + threads - 1) / threads;
  carry_combine_kernel<<<(unsigned)blocks, threads, 0, stream>>>(gathered, world, rank, rows,
                                                                 reverse, out);
  return cudaGetLastError();
}

}  // namespace fpscan
