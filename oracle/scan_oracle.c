/*
 * ORACLE — test infrastructure only.  CPU restatement of the reference
 * fpscan algorithm, used by tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline leg as the checker / CPU baseline.  Nothing in the product
 * (fpscan_b200/) links or calls this.
 *
 * Parity pinning: tests/golden/ holds vectors produced by the reference's own
 * Python (eval/baselines.py sequential_scan / parallel_scan_torch and
 * autograd through sequential_scan, as in tests/test_fpscan.py:69-87) with
 * tests/golden/make_golden.py; tests/test_oracle_golden.py checks this file
 * against them.
 *
 * Build: oracle/Makefile -> oracle/libfpscan_oracle.so (-O2, no FP
 * contraction, so the float64 loops round exactly like torch's separate
 * multiply and add in sequential_scan).
 */
#include <stdint.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* sequential_scan (eval/baselines.py:20-37): acc = gates[t]*acc + tokens[t]
 * from acc = 0, optionally over the flipped sequence. */
void oracle_scan_f64(const double* g, const double* x, double* y, int64_t rows, int64_t L,
                     int reverse) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    const double* gr = g + r * L;
    const double* xr = x + r * L;
    double* yr = y + r * L;
    double acc = 0.0;
    if (!reverse) {
      for (int64_t t = 0; t < L; ++t) {
        double p = gr[t] * acc;
        acc = p + xr[t];
        yr[t] = acc;
      }
    } else {
      for (int64_t t = L - 1; t >= 0; --t) {
        double p = gr[t] * acc;
        acc = p + xr[t];
        yr[t] = acc;
      }
    }
  }
}

/* PScan.backward (fpscan/ops.py:70-83) in float64:
 *   shifted_gates[t] = gates[t+1], shifted_gates[L-1] = 1       (ops.py:74-76)
 *   dtokens = sequential_scan(shifted_gates, grad_out, reverse)  (ops.py:77)
 *   dgates[t] = y[t-1] * dtokens[t], y[-1] = 0                   (ops.py:79-82) */
void oracle_scan_bwd_f64(const double* g, const double* y, const double* go, double* dg,
                         double* dt, int64_t rows, int64_t L) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    const double* gr = g + r * L;
    const double* yr = y + r * L;
    const double* gor = go + r * L;
    double* dgr = dg + r * L;
    double* dtr = dt + r * L;
    double acc = 0.0;
    for (int64_t t = L - 1; t >= 0; --t) {
      const double gs = (t == L - 1) ? 1.0 : gr[t + 1];
      double p = gs * acc;
      acc = p + gor[t];
      dtr[t] = acc;
      const double yp = (t == 0) ? 0.0 : yr[t - 1];
      dgr[t] = yp * acc;
    }
  }
}

/* fp32 serial forward + fused backward over `rows` rows: the CPU baseline
 * (same arithmetic as above, in float, one pass each).  Inputs/outputs fp32. */
void oracle_pscan_fwdbwd_f32(const float* g, const float* x, const float* go, float* y,
                             float* dg, float* dt, int64_t rows, int64_t L) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    const float* gr = g + r * L;
    const float* xr = x + r * L;
    const float* gor = go + r * L;
    float* yr = y + r * L;
    float* dgr = dg + r * L;
    float* dtr = dt + r * L;
    float acc = 0.f;
    for (int64_t t = 0; t < L; ++t) {
      acc = gr[t] * acc + xr[t];
      yr[t] = acc;
    }
    acc = 0.f;
    for (int64_t t = L - 1; t >= 0; --t) {
      const float gs = (t == L - 1) ? 1.f : gr[t + 1];
      acc = gs * acc + gor[t];
      dtr[t] = acc;
      dgr[t] = ((t == 0) ? 0.f : yr[t - 1]) * acc;
    }
  }
}

int oracle_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
