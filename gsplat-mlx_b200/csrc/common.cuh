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

// Can the Gaussian reach alpha >= 1/255 at any pixel centre of the tile
// whose first pixel centre is (x0, y0) and whose last is span pixels further
// on each axis (15 for a 16x16 tile)?
// sigma(d) = 0.5 (c0 dx^2 + c2 dy^2) + c1 dx dy is convex for a positive
// definite conic, so its minimum over the box of pixel-centre offsets
// [mx - x0 - span, mx - x0] x [my - y0 - span, my - y0] is 0 when the mean lies
// inside, else on an edge, where it is a 1-D quadratic minimised in closed
// form and clamped.  A Gaussian is dropped only when even that minimum
// leaves o exp(-sigma) below the threshold by a margin that covers the fp32
// rounding of the per-pixel sigma and of __expf; such a Gaussian would be
// skipped by every pixel of the tile (alpha < 1/255), so dropping it
// changes no output bit.  Conics that are not positive definite are kept,
// and so are non-finite opacities (the reference's std::min(0.99f, NaN) is
// 0.99: a NaN or +inf opacity is composited wherever sigma >= 0, a -inf one
// where its exponential underflows and -inf * 0 is NaN).
__device__ __forceinline__ bool tile_may_hit(float mx, float my, float c0, float c1, float c2,
                                             float o, float x0, float y0,
                                             float span = 15.0f) {
  if (!(fabsf(o) < INFINITY)) return true;
  if (!(c0 > 0.0f && c2 > 0.0f && c0 * c2 - c1 * c1 > 0.0f)) return true;
  const float dxl = mx - (x0 + span), dxh = mx - x0;
  const float dyl = my - (y0 + span), dyh = my - y0;
  float best = 0.0f;
  if (!(dxl <= 0.0f && dxh >= 0.0f && dyl <= 0.0f && dyh >= 0.0f)) {
    const float ry = -c1 / c2, rx = -c1 / c0;
    best = INFINITY;
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float X = e ? dxh : dxl;
      const float Y = fminf(fmaxf(ry * X, dyl), dyh);
      best = fminf(best, 0.5f * (c0 * X * X + c2 * Y * Y) + c1 * X * Y);
      const float Y2 = e ? dyh : dyl;
      const float X2 = fminf(fmaxf(rx * Y2, dxl), dxh);
      best = fminf(best, 0.5f * (c0 * X2 * X2 + c2 * Y2 * Y2) + c1 * X2 * Y2);
    }
  }
  const float xm = fmaxf(fabsf(dxl), fabsf(dxh)), ym = fmaxf(fabsf(dyl), fabsf(dyh));
  const float mag = 0.5f * (c0 * xm * xm + c2 * ym * ym) + fabsf(c1) * xm * ym;
  const float margin = 1.0e-5f * mag + 1.0e-5f;
  return o * __expf(-(best - margin)) >= (1.0f / 255.0f) * 0.998f;
}

}  // namespace gsb
