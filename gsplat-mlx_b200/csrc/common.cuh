// Shared helpers of the gsplat_b200 CUDA sources (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>

#include "../../include/gsplat_b200.h"

namespace gsb {

// Number of SMs of the current device, cached per device.
int sm_count();

// Thread-local error message behind gs_last_error().
void set_error(const char* fmt, ...);

inline cudaStream_t as_stream(gs_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

// Status of the launches just issued.
inline int launch_status(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: %s", what, cudaGetErrorString(e));
    return GS_ERR_CUDA;
  }
  return GS_OK;
}

inline int invalid(const char* msg) {
  set_error("%s", msg);
  return GS_ERR_INVALID;
}

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Grid size for a grid-stride loop over n items: enough CTAs to fill every
// SM `per_sm` times, never more than the work needs.
inline unsigned grid_for(int64_t n, int block, int per_sm = 8) {
  int64_t need = ceil_div(n, block);
  int64_t cap = static_cast<int64_t>(sm_count()) * per_sm;
  int64_t g = need < cap ? need : cap;
  return static_cast<unsigned>(g < 1 ? 1 : g);
}

// ---------------------------------------------------------------- device
__device__ __forceinline__ float4 ldg4(const float* p) {
  return __ldg(reinterpret_cast<const float4*>(p));
}

// Warp-wide sum.
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

}  // namespace gsb
