// probe.cu -- FP64 FMA-pipe probe used as the measured roofline denominator of the FDM kernel.
//
// Each thread runs 8 independent dependent-FMA chains (enough ILP to cover the DFMA latency);
// the result is written so the chains cannot be removed.  flops = 2 * 8 * iters * threads.
#include "common.cuh"

namespace f16 {
__global__ void __launch_bounds__(256) k_probe_dfma(double* __restrict__ out, int64_t iters, double a, double b) {
  double x0 = threadIdx.x * 1e-9, x1 = x0 + 1e-9, x2 = x0 + 2e-9, x3 = x0 + 3e-9;
  double x4 = x0 + 4e-9, x5 = x0 + 5e-9, x6 = x0 + 6e-9, x7 = x0 + 7e-9;
  for (int64_t i = 0; i < iters; i++) {
    x0 = fma(x0, a, b); x1 = fma(x1, a, b); x2 = fma(x2, a, b); x3 = fma(x3, a, b);
    x4 = fma(x4, a, b); x5 = fma(x5, a, b); x6 = fma(x6, a, b); x7 = fma(x7, a, b);
  }
  double s = ((x0 + x1) + (x2 + x3)) + ((x4 + x5) + (x6 + x7));
  if (s == 12345.678) out[blockIdx.x * blockDim.x + threadIdx.x] = s;   // never true; keeps the chains live
}
}  // namespace f16

// Runs blocks x 256 threads for `iters` iterations; returns the number of FP64 flops issued
// through *flops.  The caller times the launch on `stream`.
extern "C" int f16_probe_fp64(double* scratch, int64_t iters, int blocks, double* flops, f16_stream_t stream) {
  if (!scratch || iters <= 0 || blocks <= 0 || !flops) return F16_ERR_ARG;
  f16::k_probe_dfma<<<blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(scratch, iters, 0.999999, 1e-7);
  *flops = 2.0 * 8.0 * (double)iters * (double)blocks * 256.0;
  return f16::launch_status();
}
