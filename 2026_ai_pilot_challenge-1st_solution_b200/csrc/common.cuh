// common.cuh -- shared helpers of the libf16env C-ABI translation units.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include "../../include/f16env.h"

namespace f16 {

// Number of SMs of the current device (cached per device id).
inline int sm_count() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

// Map a launch result to a status (and clear the sticky-free error state).
inline int launch_status() {
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) return F16_OK;
  if (e == cudaErrorInvalidConfiguration || e == cudaErrorInvalidValue || e == cudaErrorLaunchOutOfResources)
    return F16_ERR_LAUNCH;
  return F16_ERR_CUDA;
}

inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

// Element (aircraft a, state column c) of a state buffer in either layout.
template <int LAYOUT>
struct StateRef {
  double* __restrict__ p;
  int64_t ld;
  __device__ __forceinline__ double& operator()(int64_t a, int c) const {
    return LAYOUT == F16_LAYOUT_SOA ? p[(int64_t)c * ld + a] : p[a * F16_STATE_N + c];
  }
};

}  // namespace f16
