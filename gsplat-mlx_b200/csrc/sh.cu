// Spherical harmonics (degree 0..4), forward and backward, plus the fused
// colour glue of the reference trainers.
//
// Basis and VJP math: gsplat_spherical_harmonics.cpp:116-425 (identical to
// metal/gsplat_spherical_harmonics.metal:15-308).  One thread per element;
// the degree is a template parameter so the basis is fully unrolled.  The
// ops stream the coefficient rows (K*12 bytes per element, 192 B at SH3) and
// are HBM-bound.
#include "common.cuh"

namespace gsb {
namespace {

constexpr float kC0 = 0.2820947917738781f;
constexpr float kC1 = 0.48860251190292f;

// Basis values b[0..(D+1)^2) of the unit direction (x, y, z); the zero-norm
// guard of the reference (only the DC term) is applied by the caller.
template <int D>
__device__ __forceinline__ void basis(float x, float y, float z, float* b) {
  b[0] = kC0;
  if (D < 1) return;
  b[1] = -kC1 * y;
  b[2] = kC1 * z;
  b[3] = -kC1 * x;
  if (D < 2) return;
  const float z2 = z * z;
  const float t0b = -1.092548430592079f * z;
  const float c1 = x * x - y * y, s1 = 2.0f * x * y;
  b[4] = 0.5462742152960395f * s1;
  b[5] = t0b * y;
  b[6] = 0.9461746957575601f * z2 - 0.3153915652525201f;
  b[7] = t0b * x;
  b[8] = 0.5462742152960395f * c1;
  if (D < 3) return;
  const float t0c = -2.285228997322329f * z2 + 0.4570457994644658f;
  const float t1b = 1.445305721320277f * z;
  const float c2 = x * c1 - y * s1, s2 = x * s1 + y * c1;
  b[9] = -0.5900435899266435f * s2;
  b[10] = t1b * s1;
  b[11] = t0c * y;
  b[12] = z * (1.865881662950577f * z2 - 1.119528997770346f);
  b[13] = t0c * x;
  b[14] = t1b * c1;
  b[15] = -0.5900435899266435f * c2;
  if (D < 4) return;
  const float t0d = z * (-4.683325804901025f * z2 + 2.007139630671868f);
  const float t1c = 3.31161143515146f * z2 - 0.47308734787878f;
  const float t2b = -1.770130769779931f * z;
  const float c3 = x * c2 - y * s2, s3 = x * s2 + y * c2;
  b[16] = 0.6258357354491763f * s3;
  b[17] = t2b * s2;
  b[18] = t1c * s1;
  b[19] = t0d * y;
  b[20] = 1.984313483298443f * z * b[12] - 1.006230589874905f * b[6];
  b[21] = t0d * x;
  b[22] = t1c * c1;
  b[23] = t2b * c2;
  b[24] = 0.6258357354491763f * c3;
}

// colour = sum_b basis_b * coeff_b, accumulated per degree band like the
// reference (gsplat_spherical_harmonics.cpp:189-286).
template <int D>
__device__ __forceinline__ void sh_color(const float* d, const float* co, float out[3]) {
#pragma unroll
  for (int ch = 0; ch < 3; ++ch) out[ch] = kC0 * co[ch];
  if (D < 1) return;
  const float norm = sqrtf(d[0] * d[0] + d[1] * d[1] + d[2] * d[2]);
  if (norm == 0.0f) return;
  const float x = d[0] / norm, y = d[1] / norm, z = d[2] / norm;
  float b[25];
  basis<D>(x, y, z, b);
  constexpr int bands[5] = {1, 4, 9, 16, 25};
#pragma unroll
  for (int l = 1; l <= D; ++l) {
#pragma unroll
    for (int ch = 0; ch < 3; ++ch) {
      float acc = 0.0f;
#pragma unroll
      for (int k = bands[l - 1]; k < bands[l]; ++k) acc += b[k] * co[k * 3 + ch];
      out[ch] += acc;
    }
  }
}

// gsplat_spherical_harmonics.cpp:288-425: d colour / d dir (un-normalised).
template <int D>
__device__ __forceinline__ void sh_dir_vjp(const float* d, const float* co,
                                           const float vc[3], float vd[3]) {
  vd[0] = vd[1] = vd[2] = 0.0f;
  if (D < 1) return;
  const float norm = sqrtf(d[0] * d[0] + d[1] * d[1] + d[2] * d[2]);
  if (norm == 0.0f) return;
  const float inorm = 1.0f / norm;
  const float x = d[0] * inorm, y = d[1] * inorm, z = d[2] * inorm;
  constexpr int A = (D + 1) * (D + 1);
  float dx[25], dy[25], dz[25];
#pragma unroll
  for (int i = 0; i < A; ++i) dx[i] = dy[i] = dz[i] = 0.0f;
  dx[3] = -kC1;
  dy[1] = -kC1;
  dz[2] = kC1;
  const float z2 = z * z;
  const float t0b = -1.092548430592079f * z;
  const float c1 = x * x - y * y, s1 = 2.0f * x * y;
  const float t0b_z = -1.092548430592079f;
  const float c1_x = 2.0f * x, c1_y = -2.0f * y;
  const float s1_x = 2.0f * y, s1_y = 2.0f * x;
  const float p6_z = 2.0f * 0.9461746957575601f * z;
  if (D >= 2) {
    dx[4] = 0.5462742152960395f * s1_x;
    dy[4] = 0.5462742152960395f * s1_y;
    dy[5] = t0b;
    dz[5] = t0b_z * y;
    dz[6] = p6_z;
    dx[7] = t0b;
    dz[7] = t0b_z * x;
    dx[8] = 0.5462742152960395f * c1_x;
    dy[8] = 0.5462742152960395f * c1_y;
  }
  const float t0c = -2.285228997322329f * z2 + 0.4570457994644658f;
  const float t1b = 1.445305721320277f * z;
  const float c2 = x * c1 - y * s1, s2 = x * s1 + y * c1;
  const float p12 = z * (1.865881662950577f * z2 - 1.119528997770346f);
  const float t0c_z = -2.285228997322329f * 2.0f * z;
  const float t1b_z = 1.445305721320277f;
  const float c2_x = c1 + x * c1_x - y * s1_x;
  const float c2_y = x * c1_y - s1 - y * s1_y;
  const float s2_x = s1 + x * s1_x + y * c1_x;
  const float s2_y = x * s1_y + c1 + y * c1_y;
  const float p12_z = 3.0f * 1.865881662950577f * z2 - 1.119528997770346f;
  if (D >= 3) {
    dx[9] = -0.5900435899266435f * s2_x;
    dy[9] = -0.5900435899266435f * s2_y;
    dx[10] = t1b * s1_x;
    dy[10] = t1b * s1_y;
    dz[10] = t1b_z * s1;
    dy[11] = t0c;
    dz[11] = t0c_z * y;
    dz[12] = p12_z;
    dx[13] = t0c;
    dz[13] = t0c_z * x;
    dx[14] = t1b * c1_x;
    dy[14] = t1b * c1_y;
    dz[14] = t1b_z * c1;
    dx[15] = -0.5900435899266435f * c2_x;
    dy[15] = -0.5900435899266435f * c2_y;
  }
  if (D >= 4) {
    const float t0d = z * (-4.683325804901025f * z2 + 2.007139630671868f);
    const float t1c = 3.31161143515146f * z2 - 0.47308734787878f;
    const float t2b = -1.770130769779931f * z;
    const float t0d_z = 3.0f * -4.683325804901025f * z2 + 2.007139630671868f;
    const float t1c_z = 2.0f * 3.31161143515146f * z;
    const float t2b_z = -1.770130769779931f;
    const float c3_x = c2 + x * c2_x - y * s2_x;
    const float c3_y = x * c2_y - s2 - y * s2_y;
    const float s3_x = s2 + y * c2_x + x * s2_x;
    const float s3_y = x * s2_y + c2 + y * c2_y;
    dx[16] = 0.6258357354491763f * s3_x;
    dy[16] = 0.6258357354491763f * s3_y;
    dx[17] = t2b * s2_x;
    dy[17] = t2b * s2_y;
    dz[17] = t2b_z * s2;
    dx[18] = t1c * s1_x;
    dy[18] = t1c * s1_y;
    dz[18] = t1c_z * s1;
    dy[19] = t0d;
    dz[19] = t0d_z * y;
    dz[20] = 1.984313483298443f * (p12 + z * p12_z) - 1.006230589874905f * p6_z;
    dx[21] = t0d;
    dz[21] = t0d_z * x;
    dx[22] = t1c * c1_x;
    dy[22] = t1c * c1_y;
    dz[22] = t1c_z * c1;
    dx[23] = t2b * c2_x;
    dy[23] = t2b * c2_y;
    dz[23] = t2b_z * c2;
    dx[24] = 0.6258357354491763f * c3_x;
    dy[24] = 0.6258357354491763f * c3_y;
  }
  float vn0 = 0.0f, vn1 = 0.0f, vn2 = 0.0f;
#pragma unroll
  for (int k = 1; k < A; ++k) {
    const float vb = co[k * 3] * vc[0] + co[k * 3 + 1] * vc[1] + co[k * 3 + 2] * vc[2];
    vn0 += dx[k] * vb;
    vn1 += dy[k] * vb;
    vn2 += dz[k] * vb;
  }
  const float dot = vn0 * x + vn1 * y + vn2 * z;
  vd[0] = (vn0 - dot * x) * inorm;
  vd[1] = (vn1 - dot * y) * inorm;
  vd[2] = (vn2 - dot * z) * inorm;
}

// v_coeffs row of one element: basis * v_colors for active bases, zeros for
// the rest of the K rows (the reference zero-fills its output).
template <int D>
__device__ __forceinline__ void write_vcoeffs(const float* d, const float vc[3], int K,
                                              float* __restrict__ out, bool accumulate) {
  constexpr int A = (D + 1) * (D + 1);
  float b[25];
  b[0] = kC0;
#pragma unroll
  for (int k = 1; k < A; ++k) b[k] = 0.0f;
  if (D >= 1) {
    const float norm = sqrtf(d[0] * d[0] + d[1] * d[1] + d[2] * d[2]);
    if (norm != 0.0f) basis<D>(d[0] / norm, d[1] / norm, d[2] / norm, b);
  }
#pragma unroll
  for (int k = 0; k < A; ++k)
#pragma unroll
    for (int ch = 0; ch < 3; ++ch) {
      const float v = b[k] * vc[ch];
      if (accumulate) out[k * 3 + ch] += v;
      else out[k * 3 + ch] = v;
    }
  if (!accumulate)
    for (int i = A * 3; i < K * 3; ++i) out[i] = 0.0f;
}

template <int D>
__global__ void __launch_bounds__(256) sh_fwd_kernel(int64_t n, int K,
                                                     const float* __restrict__ dirs,
                                                     const float* __restrict__ coeffs,
                                                     const uint8_t* __restrict__ masks,
                                                     float* __restrict__ colors) {
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n;
       e += (int64_t)gridDim.x * blockDim.x) {
    float c[3] = {0.0f, 0.0f, 0.0f};
    if (!masks || masks[e]) {
      const float d[3] = {__ldg(dirs + e * 3), __ldg(dirs + e * 3 + 1), __ldg(dirs + e * 3 + 2)};
      sh_color<D>(d, coeffs + e * (int64_t)K * 3, c);
    }
    colors[e * 3] = c[0];
    colors[e * 3 + 1] = c[1];
    colors[e * 3 + 2] = c[2];
  }
}

template <int D>
__global__ void __launch_bounds__(256) sh_bwd_kernel(int64_t n, int K,
                                                     const float* __restrict__ dirs,
                                                     const float* __restrict__ coeffs,
                                                     const uint8_t* __restrict__ masks,
                                                     const float* __restrict__ v_colors,
                                                     float* __restrict__ v_dirs,
                                                     float* __restrict__ v_coeffs) {
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n;
       e += (int64_t)gridDim.x * blockDim.x) {
    float* vco = v_coeffs + e * (int64_t)K * 3;
    if (masks && !masks[e]) {
      for (int i = 0; i < K * 3; ++i) vco[i] = 0.0f;
      if (v_dirs) v_dirs[e * 3] = v_dirs[e * 3 + 1] = v_dirs[e * 3 + 2] = 0.0f;
      continue;
    }
    const float d[3] = {__ldg(dirs + e * 3), __ldg(dirs + e * 3 + 1), __ldg(dirs + e * 3 + 2)};
    const float vc[3] = {__ldg(v_colors + e * 3), __ldg(v_colors + e * 3 + 1),
                         __ldg(v_colors + e * 3 + 2)};
    write_vcoeffs<D>(d, vc, K, vco, false);
    if (v_dirs) {
      float vd[3];
      sh_dir_vjp<D>(d, coeffs + e * (int64_t)K * 3, vc, vd);
      v_dirs[e * 3] = vd[0];
      v_dirs[e * 3 + 1] = vd[1];
      v_dirs[e * 3 + 2] = vd[2];
    }
  }
}

// ------------------------------------------------------------ fused glue
// scripts/test/scanner_points_training_utils.py:1005-1034 -- per Gaussian,
// looping over the C cameras: u = means - campos_c, d = u / max(|u|, 1e-8),
// colour = clip(SH(d) + 0.5, 0, 1).

__device__ __forceinline__ void campos_of(const float* __restrict__ view, float cp[3]) {
  const float R[9] = {__ldg(view + 0), __ldg(view + 1), __ldg(view + 2),
                      __ldg(view + 4), __ldg(view + 5), __ldg(view + 6),
                      __ldg(view + 8), __ldg(view + 9), __ldg(view + 10)};
  const float t[3] = {__ldg(view + 3), __ldg(view + 7), __ldg(view + 11)};
#pragma unroll
  for (int i = 0; i < 3; ++i) cp[i] = -(R[i] * t[0] + R[3 + i] * t[1] + R[6 + i] * t[2]);
}

__device__ __forceinline__ bool visible(const uint8_t* __restrict__ masks,
                                        const int32_t* __restrict__ radii, int64_t e) {
  if (masks && !masks[e]) return false;
  if (radii) {
    const int2 r = __ldg(reinterpret_cast<const int2*>(radii) + e);
    if (r.x <= 0 || r.y <= 0) return false;
  }
  return true;
}

// Backward visibility: `visible`, and with skip_zero also a non-zero colour
// cotangent (a zero cotangent contributes exactly nothing; used when the
// radii of some cameras are not at hand).
__device__ __forceinline__ bool bwd_visible(const uint8_t* __restrict__ masks,
                                            const int32_t* __restrict__ radii,
                                            const float* __restrict__ v_colors, int skip_zero,
                                            int64_t e) {
  if (!visible(masks, radii, e)) return false;
  if (!skip_zero) return true;
  const float* v = v_colors + e * 3;
  return __ldg(v) != 0.0f || __ldg(v + 1) != 0.0f || __ldg(v + 2) != 0.0f;
}

template <int D>
__global__ void __launch_bounds__(256) glue_fwd_kernel(int C, int N, int K,
                                                       const float* __restrict__ means,
                                                       const float* __restrict__ viewmats,
                                                       const float* __restrict__ coeffs,
                                                       const uint8_t* __restrict__ masks,
                                                       const int32_t* __restrict__ radii,
                                                       float* __restrict__ colors) {
  for (int64_t n = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; n < N;
       n += (int64_t)gridDim.x * blockDim.x) {
    const float m[3] = {__ldg(means + n * 3), __ldg(means + n * 3 + 1), __ldg(means + n * 3 + 2)};
    for (int c = 0; c < C; ++c) {
      const int64_t e = (int64_t)c * N + n;
      float out[3] = {0.0f, 0.0f, 0.0f};
      if (visible(masks, radii, e)) {
        float cp[3];
        campos_of(viewmats + (int64_t)c * 16, cp);
        const float u[3] = {m[0] - cp[0], m[1] - cp[1], m[2] - cp[2]};
        const float s = fmaxf(sqrtf(u[0] * u[0] + u[1] * u[1] + u[2] * u[2]), 1.0e-8f);
        const float d[3] = {u[0] / s, u[1] / s, u[2] / s};
        sh_color<D>(d, coeffs + n * (int64_t)K * 3, out);
#pragma unroll
        for (int ch = 0; ch < 3; ++ch) out[ch] = fminf(fmaxf(out[ch] + 0.5f, 0.0f), 1.0f);
      }
      colors[e * 3] = out[0];
      colors[e * 3 + 1] = out[1];
      colors[e * 3 + 2] = out[2];
    }
  }
}

// Row of viewmats for the c-th camera of the colour cotangents: with
// groups > 1 the cotangents are ordered (camera c_g of group g) as
// c = c_g * groups + g while viewmats holds group g's C / groups cameras
// contiguously (the order in which a camera-sharded step's per-camera
// all-to-alls deliver them); else c itself.
__device__ __forceinline__ int cam_row(int c, int C, int groups) {
  return groups > 1 ? (c % groups) * (C / groups) + c / groups : c;
}

template <int D>
__global__ void __launch_bounds__(256) glue_bwd_kernel(int C, int N, int K,
                                                       const float* __restrict__ means,
                                                       const float* __restrict__ viewmats,
                                                       const float* __restrict__ coeffs,
                                                       const uint8_t* __restrict__ masks,
                                                       const int32_t* __restrict__ radii,
                                                       const float* __restrict__ v_colors,
                                                       float* __restrict__ v_means,
                                                       float* __restrict__ v_coeffs,
                                                       int skip_zero, int groups) {
  for (int64_t n = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; n < N;
       n += (int64_t)gridDim.x * blockDim.x) {
    const float m[3] = {__ldg(means + n * 3), __ldg(means + n * 3 + 1), __ldg(means + n * 3 + 2)};
    const float* co = coeffs + n * (int64_t)K * 3;
    float* vco = v_coeffs + n * (int64_t)K * 3;
    float vm[3] = {0.0f, 0.0f, 0.0f};
    bool first = true;
    for (int c = 0; c < C; ++c) {
      const int64_t e = (int64_t)c * N + n;
      if (!bwd_visible(masks, radii, v_colors, skip_zero, e)) continue;
      float cp[3];
      campos_of(viewmats + (int64_t)cam_row(c, C, groups) * 16, cp);
      const float u[3] = {m[0] - cp[0], m[1] - cp[1], m[2] - cp[2]};
      const float s = sqrtf(u[0] * u[0] + u[1] * u[1] + u[2] * u[2]);
      const float mm = fmaxf(s, 1.0e-8f);
      const float d[3] = {u[0] / mm, u[1] / mm, u[2] / mm};
      float x[3];
      sh_color<D>(d, co, x);
      float vc[3];
#pragma unroll
      for (int ch = 0; ch < 3; ++ch) {
        const float v = x[ch] + 0.5f;
        vc[ch] = (v > 0.0f && v < 1.0f) ? __ldg(v_colors + e * 3 + ch) : 0.0f;
      }
      write_vcoeffs<D>(d, vc, K, vco, !first);
      first = false;
      float vd[3];
      sh_dir_vjp<D>(d, co, vc, vd);
      const float dot = vd[0] * u[0] + vd[1] * u[1] + vd[2] * u[2];
#pragma unroll
      for (int i = 0; i < 3; ++i) {
        float vu = vd[i] / mm;
        if (s > 1.0e-8f) vu -= (u[i] / s) * dot / (mm * mm);
        vm[i] += vu;
      }
    }
    if (first) {
      for (int i = 0; i < K * 3; ++i) vco[i] = 0.0f;
    } else {
      constexpr int A = (D + 1) * (D + 1);
      for (int i = A * 3; i < K * 3; ++i) vco[i] = 0.0f;
    }
    v_means[n * 3] += vm[0];
    v_means[n * 3 + 1] += vm[1];
    v_means[n * 3 + 2] += vm[2];
  }
}

// ------------------------------------------------------------ warp-staged
// Each warp owns 32 consecutive elements.  Their coefficient rows (R = 3K
// floats each, contiguous in memory) are copied into shared memory with
// whole-warp coalesced accesses -- or row by row when only a few rows are
// needed (culled Gaussians are skipped) -- at an odd row stride S, so that
// every lane can then walk its own row with conflict-free shared loads.
// Gradient rows are assembled the same way and written back with
// coalesced stores.  Used when R <= kWsMaxR (K <= 25, i.e. up to SH4).

constexpr int kWsThreads = 128;
constexpr int kWsWarps = kWsThreads / 32;
constexpr int kWsMaxR = 75;

__device__ __forceinline__ void ws_load_block(const float* __restrict__ g, int64_t e0, int cnt,
                                              int R, int S, float* sm, int lane) {
  const float* src = g + e0 * R;
  const int total = cnt * R;
  int row = 0, col = lane;
  while (col >= R) { col -= R; ++row; }
  // eight loads in flight per lane before their stores
  for (int f0 = 0; f0 < total; f0 += 32 * 8) {
    float v[8];
    int pos[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int f = f0 + lane + 32 * q;
      pos[q] = row * S + col;
      v[q] = f < total ? __ldg(src + f) : 0.0f;
      col += 32;
      while (col >= R) { col -= R; ++row; }
    }
#pragma unroll
    for (int q = 0; q < 8; ++q)
      if (f0 + lane + 32 * q < total) sm[pos[q]] = v[q];
  }
}

__device__ __forceinline__ void ws_load_rows(const float* __restrict__ g, int64_t e0, int cnt,
                                             uint32_t need, int R, int S, float* sm, int lane) {
  if (__popc(need) * 4 >= cnt * 3) {  // most rows needed: one contiguous sweep
    ws_load_block(g, e0, cnt, R, S, sm, lane);
    return;
  }
  // Eight rows per round, every load of the round issued before any store,
  // so that a warp keeps up to 24 row loads in flight instead of one.
  constexpr int kRows = 8;
  while (need) {
    int rr[kRows];
#pragma unroll
    for (int q = 0; q < kRows; ++q) {
      rr[q] = need ? __ffs(need) - 1 : -1;
      need &= need - 1;
    }
    float v[kRows][3];
#pragma unroll
    for (int q = 0; q < kRows; ++q) {
      const float* src = g + (e0 + (rr[q] < 0 ? 0 : rr[q])) * R;
#pragma unroll
      for (int k = 0; k < 3; ++k) {
        const int c = lane + 32 * k;
        v[q][k] = (rr[q] >= 0 && c < R) ? __ldg(src + c) : 0.0f;
      }
    }
#pragma unroll
    for (int q = 0; q < kRows; ++q) {
#pragma unroll
      for (int k = 0; k < 3; ++k) {
        const int c = lane + 32 * k;
        if (rr[q] >= 0 && c < R) sm[rr[q] * S + c] = v[q][k];
      }
    }
  }
}

__device__ __forceinline__ void ws_store_block(float* __restrict__ g, int64_t e0, int cnt, int R,
                                               int S, const float* sm, int lane) {
  float* dst = g + e0 * R;
  const int total = cnt * R;
  int row = 0, col = lane;
  while (col >= R) { col -= R; ++row; }
  for (int f = lane; f < total; f += 32) {
    dst[f] = sm[row * S + col];
    col += 32;
    while (col >= R) { col -= R; ++row; }
  }
}

// v_coeffs row (active bases; the caller zeroed the rest) += basis * vc.
template <int D>
__device__ __forceinline__ void add_vcoeffs(const float* d, const float vc[3], float* row) {
  constexpr int A = (D + 1) * (D + 1);
  float b[25];
  b[0] = kC0;
#pragma unroll
  for (int k = 1; k < A; ++k) b[k] = 0.0f;
  if (D >= 1) {
    const float norm = sqrtf(d[0] * d[0] + d[1] * d[1] + d[2] * d[2]);
    if (norm != 0.0f) basis<D>(d[0] / norm, d[1] / norm, d[2] / norm, b);
  }
#pragma unroll
  for (int k = 0; k < A; ++k)
#pragma unroll
    for (int ch = 0; ch < 3; ++ch) row[k * 3 + ch] += b[k] * vc[ch];
}

// ------------------------------------------------------------ vectorised
// One thread per Gaussian with its coefficient row held in registers:
// the active (D+1)^2 x 3 floats are read with back-to-back 16-byte loads
// (12 for SH3), all in flight at once, and v_coeffs rows are written with
// 16-byte stores.  Needs rows on a 16-byte boundary (K % 4 == 0 and
// aligned base pointers) and D <= 3 (the row must fit in registers); the
// other cases use the warp-staged kernels below.  The row is read once
// per Gaussian and reused for every camera.

template <int D>
__global__ void __launch_bounds__(256) glue_fwd_vec_kernel(
    int C, int N, int K, const float* __restrict__ means, const float* __restrict__ viewmats,
    const float* __restrict__ coeffs, const uint8_t* __restrict__ masks,
    const int32_t* __restrict__ radii, float* __restrict__ colors) {
  constexpr int A = (D + 1) * (D + 1);
  constexpr int NV = (A * 3 + 3) / 4;
  for (int64_t n = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; n < N;
       n += (int64_t)gridDim.x * blockDim.x) {
    bool any = false;
    for (int c = 0; c < C; ++c) any |= visible(masks, radii, (int64_t)c * N + n);
    float co[NV * 4];
    float m[3] = {0.0f, 0.0f, 0.0f};
    if (any) {
      const float4* row = reinterpret_cast<const float4*>(coeffs + n * (int64_t)K * 3);
#pragma unroll
      for (int v = 0; v < NV; ++v) {
        const float4 q = __ldg(row + v);
        co[4 * v] = q.x;
        co[4 * v + 1] = q.y;
        co[4 * v + 2] = q.z;
        co[4 * v + 3] = q.w;
      }
      m[0] = __ldg(means + n * 3);
      m[1] = __ldg(means + n * 3 + 1);
      m[2] = __ldg(means + n * 3 + 2);
    }
    for (int c = 0; c < C; ++c) {
      const int64_t e = (int64_t)c * N + n;
      float out[3] = {0.0f, 0.0f, 0.0f};
      if (any && visible(masks, radii, e)) {
        float cp[3];
        campos_of(viewmats + (int64_t)c * 16, cp);
        const float u[3] = {m[0] - cp[0], m[1] - cp[1], m[2] - cp[2]};
        const float s = fmaxf(sqrtf(u[0] * u[0] + u[1] * u[1] + u[2] * u[2]), 1.0e-8f);
        const float d[3] = {u[0] / s, u[1] / s, u[2] / s};
        sh_color<D>(d, co, out);
#pragma unroll
        for (int ch = 0; ch < 3; ++ch) out[ch] = fminf(fmaxf(out[ch] + 0.5f, 0.0f), 1.0f);
      }
      colors[e * 3] = out[0];
      colors[e * 3 + 1] = out[1];
      colors[e * 3 + 2] = out[2];
    }
  }
}

// ACC = false (one camera): the v_coeffs row is written as it is formed
// (16-byte stores), which keeps the register count low enough for latency
// hiding.  ACC = true (several cameras): the row is summed over the cameras
// in registers and written once.
// One Gaussian that some camera sees: its coefficient row in registers,
// every visible camera's colour cotangent through the clamp, the basis and
// the direction VJP; v_coeffs row written (accumulated in registers when
// ACC, else read-modify-written camera by camera), zeros past the degree's
// bases, the SH part of v_means added.
template <int D, bool ACC>
__device__ __forceinline__ void glue_bwd_vec_one(
    int64_t n, int C, int N, int K, const float* __restrict__ means,
    const float* __restrict__ viewmats, const float* __restrict__ coeffs,
    const uint8_t* __restrict__ masks, const int32_t* __restrict__ radii,
    const float* __restrict__ v_colors, float* __restrict__ v_means, float* __restrict__ v_coeffs,
    int skip_zero, int groups) {
  constexpr int A = (D + 1) * (D + 1);
  constexpr int NV = (A * 3 + 3) / 4;
  float4* out = reinterpret_cast<float4*>(v_coeffs + n * (int64_t)K * 3);
  float co[NV * 4];
  const float4* row = reinterpret_cast<const float4*>(coeffs + n * (int64_t)K * 3);
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    const float4 q = __ldg(row + v);
    co[4 * v] = q.x;
    co[4 * v + 1] = q.y;
    co[4 * v + 2] = q.z;
    co[4 * v + 3] = q.w;
  }
  const float m[3] = {__ldg(means + n * 3), __ldg(means + n * 3 + 1), __ldg(means + n * 3 + 2)};
  float vm[3] = {0.0f, 0.0f, 0.0f};
  float acc[ACC ? NV * 4 : 1];
#pragma unroll
  for (int i = 0; i < (ACC ? NV * 4 : 1); ++i) acc[i] = 0.0f;
  bool first = true;
  for (int c = 0; c < C; ++c) {
    const int64_t e = (int64_t)c * N + n;
    if (!bwd_visible(masks, radii, v_colors, skip_zero, e)) continue;
    float cp[3];
    campos_of(viewmats + (int64_t)cam_row(c, C, groups) * 16, cp);
    const float u[3] = {m[0] - cp[0], m[1] - cp[1], m[2] - cp[2]};
    const float s = sqrtf(u[0] * u[0] + u[1] * u[1] + u[2] * u[2]);
    const float mm = fmaxf(s, 1.0e-8f);
    const float d[3] = {u[0] / mm, u[1] / mm, u[2] / mm};
    float x[3];
    sh_color<D>(d, co, x);
    float vc[3];
#pragma unroll
    for (int ch = 0; ch < 3; ++ch) {
      const float v = x[ch] + 0.5f;
      vc[ch] = (v > 0.0f && v < 1.0f) ? __ldg(v_colors + e * 3 + ch) : 0.0f;
    }
    // basis (the reference's zero-norm guard keeps only the DC term)
    float b[NV * 4 / 3 + 1];
#pragma unroll
    for (int k = 0; k < NV * 4 / 3 + 1; ++k) b[k] = 0.0f;
    b[0] = kC0;
    if (D >= 1) {
      const float norm = sqrtf(d[0] * d[0] + d[1] * d[1] + d[2] * d[2]);
      if (norm != 0.0f) basis<D>(d[0] / norm, d[1] / norm, d[2] / norm, b);
    }
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      float q[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const int idx = 4 * v + t;  // (basis idx / 3, channel idx % 3)
        q[t] = idx < A * 3 ? b[idx / 3] * vc[idx % 3] : 0.0f;
      }
      if (ACC) {
#pragma unroll
        for (int t = 0; t < 4; ++t) acc[(ACC ? 4 * v + t : 0)] += q[t];
      } else {
        float4 val = make_float4(q[0], q[1], q[2], q[3]);
        if (!first) {
          const float4 o = out[v];
          val.x += o.x;
          val.y += o.y;
          val.z += o.z;
          val.w += o.w;
        }
        out[v] = val;
      }
    }
    first = false;
    float vd[3];
    sh_dir_vjp<D>(d, co, vc, vd);
    const float dot = vd[0] * u[0] + vd[1] * u[1] + vd[2] * u[2];
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      float vu = vd[i] / mm;
      if (s > 1.0e-8f) vu -= (u[i] / s) * dot / (mm * mm);
      vm[i] += vu;
    }
  }
  if (ACC) {
#pragma unroll
    for (int v = 0; v < NV; ++v)
      out[v] = make_float4(acc[(ACC ? 4 * v : 0)], acc[(ACC ? 4 * v + 1 : 0)],
                           acc[(ACC ? 4 * v + 2 : 0)], acc[(ACC ? 4 * v + 3 : 0)]);
  }
  v_means[n * 3] += vm[0];
  v_means[n * 3 + 1] += vm[1];
  v_means[n * 3 + 2] += vm[2];
  for (int v = NV; v < K * 3 / 4; ++v) out[v] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
}

// Each warp walks chunks of 32 Gaussians: the ones no camera sees get their
// zero v_coeffs row at once; the others go to a per-warp queue in shared
// memory and are processed 32 at a time, one per lane, so that the heavy
// per-camera work runs on full warps (a third of the Gaussians are visible
// at config 3: one Gaussian per thread left two thirds of the lanes idle).
// The one-camera form is capped at 128 registers (4 CTAs per SM; the
// multi-camera form, with its register accumulators, is not: it would
// spill).  Measured: config 3 0.101 -> 0.096 ms, config 4 6.2 -> 5.7 ms.
constexpr int kGlueBwdWarps = 4;

template <int D, bool ACC>
__global__ void __launch_bounds__(32 * kGlueBwdWarps, ACC ? 3 : 4) glue_bwd_vec_kernel(
    int C, int N, int K, const float* __restrict__ means, const float* __restrict__ viewmats,
    const float* __restrict__ coeffs, const uint8_t* __restrict__ masks,
    const int32_t* __restrict__ radii, const float* __restrict__ v_colors,
    float* __restrict__ v_means, float* __restrict__ v_coeffs, int skip_zero, int groups) {
  __shared__ int s_q[kGlueBwdWarps][64];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int* q = s_q[warp];
  int qn = 0;
  const int64_t chunks = ((int64_t)N + 31) / 32;
  for (int64_t ch = (int64_t)blockIdx.x * kGlueBwdWarps + warp; ch < chunks;
       ch += (int64_t)gridDim.x * kGlueBwdWarps) {
    const int64_t n = ch * 32 + lane;
    bool any = false;
    if (n < N) {
      for (int c = 0; c < C; ++c)
        any |= bwd_visible(masks, radii, v_colors, skip_zero, (int64_t)c * N + n);
    }
    const unsigned bal = __ballot_sync(0xffffffffu, any);
    {
      // zero rows of the chunk's Gaussians that no camera sees: the chunk's
      // rows are contiguous, so the warp stores them together (512 B per
      // store instruction) rather than one row per lane
      const int per = K * 3 / 4;  // float4 per row
      const int rows = (int)min((int64_t)32, (int64_t)N - ch * 32);
      float4* base = reinterpret_cast<float4*>(v_coeffs + ch * 32 * (int64_t)K * 3);
      for (int f = lane; f < rows * per; f += 32)
        if (!((bal >> (f / per)) & 1u)) base[f] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
    if (any) q[qn + __popc(bal & ((1u << lane) - 1u))] = (int)n;
    qn += __popc(bal);
    __syncwarp();
    if (qn >= 32) {
      glue_bwd_vec_one<D, ACC>(q[qn - 32 + lane], C, N, K, means, viewmats, coeffs, masks, radii,
                               v_colors, v_means, v_coeffs, skip_zero, groups);
      qn -= 32;
      __syncwarp();
    }
  }
  if (lane < qn)
    glue_bwd_vec_one<D, ACC>(q[lane], C, N, K, means, viewmats, coeffs, masks, radii, v_colors,
                             v_means, v_coeffs, skip_zero, groups);
}

template <int D>
__global__ void __launch_bounds__(kWsThreads) glue_fwd_ws_kernel(
    int C, int N, int K, const float* __restrict__ means, const float* __restrict__ viewmats,
    const float* __restrict__ coeffs, const uint8_t* __restrict__ masks,
    const int32_t* __restrict__ radii, float* __restrict__ colors) {
  extern __shared__ float smem[];
  const int R = K * 3, S = R | 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* sm = smem + warp * 32 * S;
  const int64_t chunks = (N + 31) / 32;
  for (int64_t ch = (int64_t)blockIdx.x * kWsWarps + warp; ch < chunks;
       ch += (int64_t)gridDim.x * kWsWarps) {
    const int64_t e0 = ch * 32;
    const int cnt = (int)(N - e0 < 32 ? N - e0 : 32);
    const int64_t n = e0 + lane;
    const bool live = lane < cnt;
    bool any = false;
    for (int c = 0; c < C && live; ++c) any |= visible(masks, radii, (int64_t)c * N + n);
    const uint32_t need = __ballot_sync(0xffffffffu, any);
    ws_load_rows(coeffs, e0, cnt, need, R, S, sm, lane);
    __syncwarp();
    float m[3] = {0.f, 0.f, 0.f};
    if (live) {
      m[0] = __ldg(means + n * 3);
      m[1] = __ldg(means + n * 3 + 1);
      m[2] = __ldg(means + n * 3 + 2);
    }
    for (int c = 0; c < C; ++c) {
      if (!live) break;
      const int64_t e = (int64_t)c * N + n;
      float out[3] = {0.0f, 0.0f, 0.0f};
      if (visible(masks, radii, e)) {
        float cp[3];
        campos_of(viewmats + (int64_t)c * 16, cp);
        const float u[3] = {m[0] - cp[0], m[1] - cp[1], m[2] - cp[2]};
        const float s = fmaxf(sqrtf(u[0] * u[0] + u[1] * u[1] + u[2] * u[2]), 1.0e-8f);
        const float d[3] = {u[0] / s, u[1] / s, u[2] / s};
        sh_color<D>(d, sm + lane * S, out);
#pragma unroll
        for (int k = 0; k < 3; ++k) out[k] = fminf(fmaxf(out[k] + 0.5f, 0.0f), 1.0f);
      }
      colors[e * 3] = out[0];
      colors[e * 3 + 1] = out[1];
      colors[e * 3 + 2] = out[2];
    }
    __syncwarp();
  }
}

template <int D>
__global__ void __launch_bounds__(kWsThreads) glue_bwd_ws_kernel(
    int C, int N, int K, const float* __restrict__ means, const float* __restrict__ viewmats,
    const float* __restrict__ coeffs, const uint8_t* __restrict__ masks,
    const int32_t* __restrict__ radii, const float* __restrict__ v_colors,
    float* __restrict__ v_means, float* __restrict__ v_coeffs, int skip_zero, int groups) {
  extern __shared__ float smem[];
  const int R = K * 3, S = R | 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* sm = smem + warp * 64 * S;   // coefficient rows
  float* sv = sm + 32 * S;            // gradient rows
  const int64_t chunks = (N + 31) / 32;
  for (int64_t ch = (int64_t)blockIdx.x * kWsWarps + warp; ch < chunks;
       ch += (int64_t)gridDim.x * kWsWarps) {
    const int64_t e0 = ch * 32;
    const int cnt = (int)(N - e0 < 32 ? N - e0 : 32);
    const int64_t n = e0 + lane;
    const bool live = lane < cnt;
    bool any = false;
    for (int c = 0; c < C && live; ++c) any |= bwd_visible(masks, radii, v_colors, skip_zero, (int64_t)c * N + n);
    const uint32_t need = __ballot_sync(0xffffffffu, any);
    ws_load_rows(coeffs, e0, cnt, need, R, S, sm, lane);
    float* myv = sv + lane * S;
    for (int j = 0; j < R; ++j) myv[j] = 0.0f;
    __syncwarp();
    float vm[3] = {0.0f, 0.0f, 0.0f};
    if (any) {
      const float m[3] = {__ldg(means + n * 3), __ldg(means + n * 3 + 1), __ldg(means + n * 3 + 2)};
      const float* co = sm + lane * S;
      for (int c = 0; c < C; ++c) {
        const int64_t e = (int64_t)c * N + n;
        if (!bwd_visible(masks, radii, v_colors, skip_zero, e)) continue;
        float cp[3];
        campos_of(viewmats + (int64_t)cam_row(c, C, groups) * 16, cp);
        const float u[3] = {m[0] - cp[0], m[1] - cp[1], m[2] - cp[2]};
        const float s = sqrtf(u[0] * u[0] + u[1] * u[1] + u[2] * u[2]);
        const float mm = fmaxf(s, 1.0e-8f);
        const float d[3] = {u[0] / mm, u[1] / mm, u[2] / mm};
        float x[3];
        sh_color<D>(d, co, x);
        float vc[3];
#pragma unroll
        for (int k = 0; k < 3; ++k) {
          const float v = x[k] + 0.5f;
          vc[k] = (v > 0.0f && v < 1.0f) ? __ldg(v_colors + e * 3 + k) : 0.0f;
        }
        add_vcoeffs<D>(d, vc, myv);
        float vd[3];
        sh_dir_vjp<D>(d, co, vc, vd);
        const float dot = vd[0] * u[0] + vd[1] * u[1] + vd[2] * u[2];
#pragma unroll
        for (int i = 0; i < 3; ++i) {
          float vu = vd[i] / mm;
          if (s > 1.0e-8f) vu -= (u[i] / s) * dot / (mm * mm);
          vm[i] += vu;
        }
      }
    }
    __syncwarp();
    ws_store_block(v_coeffs, e0, cnt, R, S, sv, lane);
    if (live) {
      v_means[n * 3] += vm[0];
      v_means[n * 3 + 1] += vm[1];
      v_means[n * 3 + 2] += vm[2];
    }
    __syncwarp();
  }
}

template <int D>
__global__ void __launch_bounds__(kWsThreads) sh_fwd_ws_kernel(int64_t n, int K,
                                                               const float* __restrict__ dirs,
                                                               const float* __restrict__ coeffs,
                                                               const uint8_t* __restrict__ masks,
                                                               float* __restrict__ colors) {
  extern __shared__ float smem[];
  const int R = K * 3, S = R | 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* sm = smem + warp * 32 * S;
  const int64_t chunks = (n + 31) / 32;
  for (int64_t ch = (int64_t)blockIdx.x * kWsWarps + warp; ch < chunks;
       ch += (int64_t)gridDim.x * kWsWarps) {
    const int64_t e0 = ch * 32;
    const int cnt = (int)(n - e0 < 32 ? n - e0 : 32);
    const int64_t e = e0 + lane;
    const bool on = lane < cnt && (!masks || masks[e]);
    ws_load_rows(coeffs, e0, cnt, __ballot_sync(0xffffffffu, on), R, S, sm, lane);
    __syncwarp();
    if (lane < cnt) {
      float c[3] = {0.0f, 0.0f, 0.0f};
      if (on) {
        const float d[3] = {__ldg(dirs + e * 3), __ldg(dirs + e * 3 + 1), __ldg(dirs + e * 3 + 2)};
        sh_color<D>(d, sm + lane * S, c);
      }
      colors[e * 3] = c[0];
      colors[e * 3 + 1] = c[1];
      colors[e * 3 + 2] = c[2];
    }
    __syncwarp();
  }
}

template <int D>
__global__ void __launch_bounds__(kWsThreads) sh_bwd_ws_kernel(
    int64_t n, int K, const float* __restrict__ dirs, const float* __restrict__ coeffs,
    const uint8_t* __restrict__ masks, const float* __restrict__ v_colors,
    float* __restrict__ v_dirs, float* __restrict__ v_coeffs) {
  extern __shared__ float smem[];
  const int R = K * 3, S = R | 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* sm = smem + warp * 64 * S;
  float* sv = sm + 32 * S;
  const int64_t chunks = (n + 31) / 32;
  for (int64_t ch = (int64_t)blockIdx.x * kWsWarps + warp; ch < chunks;
       ch += (int64_t)gridDim.x * kWsWarps) {
    const int64_t e0 = ch * 32;
    const int cnt = (int)(n - e0 < 32 ? n - e0 : 32);
    const int64_t e = e0 + lane;
    const bool on = lane < cnt && (!masks || masks[e]);
    // coefficient rows are only read for v_dirs
    ws_load_rows(coeffs, e0, cnt, v_dirs ? __ballot_sync(0xffffffffu, on) : 0u, R, S, sm, lane);
    float* myv = sv + lane * S;
    for (int j = 0; j < R; ++j) myv[j] = 0.0f;
    __syncwarp();
    if (on) {
      const float d[3] = {__ldg(dirs + e * 3), __ldg(dirs + e * 3 + 1), __ldg(dirs + e * 3 + 2)};
      const float vc[3] = {__ldg(v_colors + e * 3), __ldg(v_colors + e * 3 + 1),
                           __ldg(v_colors + e * 3 + 2)};
      add_vcoeffs<D>(d, vc, myv);
      if (v_dirs) {
        float vd[3];
        sh_dir_vjp<D>(d, sm + lane * S, vc, vd);
        v_dirs[e * 3] = vd[0];
        v_dirs[e * 3 + 1] = vd[1];
        v_dirs[e * 3 + 2] = vd[2];
      }
    } else if (lane < cnt && v_dirs) {
      v_dirs[e * 3] = v_dirs[e * 3 + 1] = v_dirs[e * 3 + 2] = 0.0f;
    }
    __syncwarp();
    ws_store_block(v_coeffs, e0, cnt, R, S, sv, lane);
    __syncwarp();
  }
}

// Launch helper of the staged kernels: `rows` row buffers of 32 x S floats
// per warp.
template <typename Kern>
int ws_launch(Kern kernel, int64_t elems, int K, int rows, cudaStream_t s, const char* what,
              void** args) {
  const int S = (K * 3) | 1;
  const size_t smem = sizeof(float) * (size_t)kWsWarps * rows * 32 * S;
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  const int64_t chunks = (elems + 31) / 32;
  const unsigned grid = grid_for(chunks, kWsWarps, 8);
  if (cudaLaunchKernel((const void*)kernel, dim3(grid), dim3(kWsThreads), args, smem, s) !=
      cudaSuccess)
    return launch_status(what);
  return launch_status(what);
}

template <template <int> class Launch, typename... Args>
int by_degree(int degree, Args... args) {
  switch (degree) {
    case 0: return Launch<0>::run(args...);
    case 1: return Launch<1>::run(args...);
    case 2: return Launch<2>::run(args...);
    case 3: return Launch<3>::run(args...);
    case 4: return Launch<4>::run(args...);
    default: return invalid("spherical_harmonics supports degree 0..4.");
  }
}

template <int D>
struct FwdL {
  static int run(const gs_sh_params* p, const float* dirs, const float* coeffs,
                 const uint8_t* masks, float* colors, cudaStream_t s) {
    if (p->K * 3 <= kWsMaxR) {
      int64_t n = p->n;
      int K = p->K;
      const uint8_t* mk = p->use_masks ? masks : nullptr;
      void* args[] = {&n, &K, &dirs, &coeffs, &mk, &colors};
      return ws_launch(sh_fwd_ws_kernel<D>, n, K, 1, s, "sh_fwd", args);
    }
    sh_fwd_kernel<D><<<grid_for(p->n, 256), 256, 0, s>>>(p->n, p->K, dirs, coeffs,
                                                         p->use_masks ? masks : nullptr, colors);
    return launch_status("sh_fwd");
  }
};

template <int D>
struct BwdL {
  static int run(const gs_sh_params* p, const float* dirs, const float* coeffs,
                 const uint8_t* masks, const float* v_colors, float* v_dirs, float* v_coeffs,
                 cudaStream_t s) {
    if (p->K * 3 <= kWsMaxR) {
      int64_t n = p->n;
      int K = p->K;
      const uint8_t* mk = p->use_masks ? masks : nullptr;
      void* args[] = {&n, &K, &dirs, &coeffs, &mk, &v_colors, &v_dirs, &v_coeffs};
      return ws_launch(sh_bwd_ws_kernel<D>, n, K, 2, s, "sh_bwd", args);
    }
    sh_bwd_kernel<D><<<grid_for(p->n, 256), 256, 0, s>>>(
        p->n, p->K, dirs, coeffs, p->use_masks ? masks : nullptr, v_colors, v_dirs, v_coeffs);
    return launch_status("sh_bwd");
  }
};

// The vectorised glue kernels apply: SH degree <= 3 and 16-byte rows.
template <int D>
bool vec_ok(int K, const float* a, const float* b) {
  return D <= 3 && K % 4 == 0 && (reinterpret_cast<uintptr_t>(a) & 15) == 0 &&
         (reinterpret_cast<uintptr_t>(b) & 15) == 0;
}

template <int D>
struct GlueFwdL {
  static int run(const gs_sh_glue_params* p, const float* means, const float* viewmats,
                 const float* coeffs, const uint8_t* masks, const int32_t* radii, float* colors,
                 cudaStream_t s) {
    if (vec_ok<D>(p->K, coeffs, nullptr)) {
      glue_fwd_vec_kernel<(D < 3 ? D : 3)><<<grid_for(p->N, 256), 256, 0, s>>>(
          p->C, p->N, p->K, means, viewmats, coeffs, p->use_masks ? masks : nullptr, radii,
          colors);
      return launch_status("sh_glue_fwd");
    }
    if (p->K * 3 <= kWsMaxR) {
      int C = p->C, N = p->N, K = p->K;
      const uint8_t* mk = p->use_masks ? masks : nullptr;
      void* args[] = {&C, &N, &K, &means, &viewmats, &coeffs, &mk, &radii, &colors};
      return ws_launch(glue_fwd_ws_kernel<D>, N, K, 1, s, "sh_glue_fwd", args);
    }
    glue_fwd_kernel<D><<<grid_for(p->N, 256), 256, 0, s>>>(
        p->C, p->N, p->K, means, viewmats, coeffs, p->use_masks ? masks : nullptr, radii, colors);
    return launch_status("sh_glue_fwd");
  }
};

template <int D>
struct GlueBwdL {
  static int run(const gs_sh_glue_params* p, const float* means, const float* viewmats,
                 const float* coeffs, const uint8_t* masks, const int32_t* radii,
                 const float* v_colors, float* v_means, float* v_coeffs, cudaStream_t s) {
    if (vec_ok<D>(p->K, coeffs, v_coeffs)) {
      constexpr int DV = D < 3 ? D : 3;
      auto kern = p->C > 1 ? glue_bwd_vec_kernel<DV, true> : glue_bwd_vec_kernel<DV, false>;
      kern<<<grid_for(p->N, 32 * kGlueBwdWarps), 32 * kGlueBwdWarps, 0, s>>>(
          p->C, p->N, p->K, means, viewmats, coeffs, p->use_masks ? masks : nullptr, radii,
          v_colors, v_means, v_coeffs, p->skip_zero_cotangents, p->camera_groups);
      return launch_status("sh_glue_bwd");
    }
    if (p->K * 3 <= kWsMaxR) {
      int C = p->C, N = p->N, K = p->K;
      const uint8_t* mk = p->use_masks ? masks : nullptr;
      int skip = p->skip_zero_cotangents, groups = p->camera_groups;
      void* args[] = {&C, &N, &K, &means, &viewmats, &coeffs, &mk, &radii, &v_colors, &v_means,
                      &v_coeffs, &skip, &groups};
      return ws_launch(glue_bwd_ws_kernel<D>, N, K, 2, s, "sh_glue_bwd", args);
    }
    glue_bwd_kernel<D><<<grid_for(p->N, 256), 256, 0, s>>>(p->C, p->N, p->K, means, viewmats,
                                                           coeffs, p->use_masks ? masks : nullptr,
                                                           radii, v_colors, v_means, v_coeffs,
                                                           p->skip_zero_cotangents,
                                                           p->camera_groups);
    return launch_status("sh_glue_bwd");
  }
};

int check_sh(const gs_sh_params* p) {
  if (!p || p->n < 0) return invalid("spherical_harmonics: bad params");
  if (p->degrees_to_use < 0 || p->degrees_to_use > 4)
    return invalid("spherical_harmonics_forward supports degree 0..4.");
  if (p->K < (p->degrees_to_use + 1) * (p->degrees_to_use + 1))
    return invalid("coeffs has fewer SH bases than degrees_to_use requires.");
  return GS_OK;
}

int check_glue(const gs_sh_glue_params* p) {
  if (!p || p->C < 0 || p->N < 0) return invalid("sh_glue: bad params");
  if (p->camera_groups > 1 && p->C % p->camera_groups)
    return invalid("sh_glue: the camera count must be a multiple of camera_groups");
  if (p->degrees_to_use < 0 || p->degrees_to_use > 4)
    return invalid("sh_glue: degree must be 0..4");
  if (p->K < (p->degrees_to_use + 1) * (p->degrees_to_use + 1))
    return invalid("sh_glue: coeffs has fewer SH bases than the degree requires");
  return GS_OK;
}

}  // namespace
}  // namespace gsb

extern "C" int gs_sh_fwd(const gs_sh_params* p, const float* dirs, const float* coeffs,
                         const uint8_t* masks, float* colors, gs_stream_t stream) {
  using namespace gsb;
  if (int rc = check_sh(p)) return rc;
  if (p->n == 0) return GS_OK;
  if (!dirs || !coeffs || !colors || (p->use_masks && !masks))
    return invalid("sh_fwd: missing buffer");
  return by_degree<FwdL>(p->degrees_to_use, p, dirs, coeffs, masks, colors, as_stream(stream));
}

extern "C" int gs_sh_bwd(const gs_sh_params* p, const float* dirs, const float* coeffs,
                         const uint8_t* masks, const float* v_colors, float* v_dirs,
                         float* v_coeffs, gs_stream_t stream) {
  using namespace gsb;
  if (int rc = check_sh(p)) return rc;
  if (p->n == 0) return GS_OK;
  if (!dirs || !coeffs || !v_colors || !v_coeffs || (p->use_masks && !masks))
    return invalid("sh_bwd: missing buffer");
  return by_degree<BwdL>(p->degrees_to_use, p, dirs, coeffs, masks, v_colors, v_dirs, v_coeffs,
                         as_stream(stream));
}

extern "C" int gs_sh_glue_fwd(const gs_sh_glue_params* p, const float* means,
                              const float* viewmats, const float* coeffs, const uint8_t* masks,
                              const int32_t* radii, float* colors, gs_stream_t stream) {
  using namespace gsb;
  if (int rc = check_glue(p)) return rc;
  if ((int64_t)p->C * p->N == 0) return GS_OK;
  if (!means || !viewmats || !coeffs || !colors || (p->use_masks && !masks))
    return invalid("sh_glue_fwd: missing buffer");
  if (reinterpret_cast<uintptr_t>(radii) % 8) return invalid("sh_glue_fwd: radii must be 8-byte aligned");
  return by_degree<GlueFwdL>(p->degrees_to_use, p, means, viewmats, coeffs, masks, radii, colors,
                             as_stream(stream));
}

extern "C" int gs_sh_glue_bwd(const gs_sh_glue_params* p, const float* means,
                              const float* viewmats, const float* coeffs, const uint8_t* masks,
                              const int32_t* radii, const float* v_colors, float* v_means_accum,
                              float* v_coeffs, gs_stream_t stream) {
  using namespace gsb;
  if (int rc = check_glue(p)) return rc;
  if (p->N == 0) return GS_OK;
  if (!means || !viewmats || !coeffs || !v_colors || !v_means_accum || !v_coeffs ||
      (p->use_masks && !masks))
    return invalid("sh_glue_bwd: missing buffer");
  if (reinterpret_cast<uintptr_t>(radii) % 8) return invalid("sh_glue_bwd: radii must be 8-byte aligned");
  return by_degree<GlueBwdL>(p->degrees_to_use, p, means, viewmats, coeffs, masks, radii,
                             v_colors, v_means_accum, v_coeffs, as_stream(stream));
}
