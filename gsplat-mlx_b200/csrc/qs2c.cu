// quat/scale -> covariance / precision, forward and backward.
//
// Math: gsplat_quat_scale_to_covar.cpp:103-333 (CPU) and
// metal/gsplat_quat_scale_to_covar.metal:16-321 (GPU).  One thread per
// (quat, scale) pair; the op is HBM-bound (28 B in, 24/48 B out per pair).
// A zero quaternion yields NaN as on the Metal path (the CPU path throws).
#include "common.cuh"

namespace gsb {
namespace {

struct M3 {
  float v[9];
};

__device__ __forceinline__ M3 rotmat(float w, float x, float y, float z) {
  const float norm = sqrtf(w * w + x * x + y * y + z * z);
  w /= norm;
  x /= norm;
  y /= norm;
  z /= norm;
  const float x2 = x * x, y2 = y * y, z2 = z * z;
  const float xy = x * y, xz = x * z, yz = y * z;
  const float wx = w * x, wy = w * y, wz = w * z;
  M3 r;
  r.v[0] = 1.0f - 2.0f * (y2 + z2);
  r.v[1] = 2.0f * (xy - wz);
  r.v[2] = 2.0f * (xz + wy);
  r.v[3] = 2.0f * (xy + wz);
  r.v[4] = 1.0f - 2.0f * (x2 + z2);
  r.v[5] = 2.0f * (yz - wx);
  r.v[6] = 2.0f * (xz - wy);
  r.v[7] = 2.0f * (yz + wx);
  r.v[8] = 1.0f - 2.0f * (x2 + y2);
  return r;
}

// R diag(s*s) R^T  (s already inverted for the precision)
__device__ __forceinline__ M3 rss(const M3& r, const float s[3]) {
  M3 o;
  const float ss[3] = {s[0] * s[0], s[1] * s[1], s[2] * s[2]};
#pragma unroll
  for (int i = 0; i < 3; ++i)
#pragma unroll
    for (int j = 0; j < 3; ++j)
      o.v[i * 3 + j] = r.v[i * 3] * ss[0] * r.v[j * 3] + r.v[i * 3 + 1] * ss[1] * r.v[j * 3 + 1] +
                       r.v[i * 3 + 2] * ss[2] * r.v[j * 3 + 2];
  return o;
}

__device__ __forceinline__ void store(const M3& m, bool triu, float* out) {
  if (triu) {
    out[0] = m.v[0];
    out[1] = m.v[1];
    out[2] = m.v[2];
    out[3] = m.v[4];
    out[4] = m.v[5];
    out[5] = m.v[8];
  } else {
#pragma unroll
    for (int i = 0; i < 9; ++i) out[i] = m.v[i];
  }
}

__global__ void __launch_bounds__(256) qs2c_fwd_kernel(int64_t n, const float* __restrict__ quats,
                                                       const float* __restrict__ scales,
                                                       float* __restrict__ covars,
                                                       float* __restrict__ precis, int compute_covar,
                                                       int compute_preci, int triu) {
  const int stride = triu ? 6 : 9;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n;
       e += (int64_t)gridDim.x * blockDim.x) {
    const float* q = quats + e * 4;
    const M3 r = rotmat(__ldg(q), __ldg(q + 1), __ldg(q + 2), __ldg(q + 3));
    float s[3] = {__ldg(scales + e * 3), __ldg(scales + e * 3 + 1), __ldg(scales + e * 3 + 2)};
    if (compute_covar) store(rss(r, s), triu, covars + e * stride);
    if (compute_preci) {
      float si[3] = {1.0f / s[0], 1.0f / s[1], 1.0f / s[2]};
      store(rss(r, si), triu, precis + e * stride);
    }
  }
}

// Symmetric split of the cotangent, gsplat_quat_scale_to_covar.cpp:215-236.
__device__ __forceinline__ M3 cot_matrix(bool triu, const float* c) {
  M3 o;
  if (triu) {
    o.v[0] = c[0];
    o.v[1] = 0.5f * c[1];
    o.v[2] = 0.5f * c[2];
    o.v[3] = 0.5f * c[1];
    o.v[4] = c[3];
    o.v[5] = 0.5f * c[4];
    o.v[6] = 0.5f * c[2];
    o.v[7] = 0.5f * c[4];
    o.v[8] = c[5];
  } else {
#pragma unroll
    for (int i = 0; i < 9; ++i) o.v[i] = c[i];
  }
  return o;
}

// gsplat_quat_scale_to_covar.cpp:238-276: d R(q/|q|) / d q applied to g.
__device__ __forceinline__ void rotmat_vjp(float w, float x, float y, float z, const M3& g,
                                           float vq[4]) {
  const float inv = 1.0f / sqrtf(w * w + x * x + y * y + z * z);
  w *= inv;
  x *= inv;
  y *= inv;
  z *= inv;
  const float* G = g.v;
  const float v1 = 2.0f * y * G[1] + 2.0f * z * G[2] + 2.0f * y * G[3] - 4.0f * x * G[4] -
                   2.0f * w * G[5] + 2.0f * z * G[6] + 2.0f * w * G[7] - 4.0f * x * G[8];
  const float v2 = -4.0f * y * G[0] + 2.0f * x * G[1] + 2.0f * w * G[2] + 2.0f * x * G[3] +
                   2.0f * z * G[5] - 2.0f * w * G[6] + 2.0f * z * G[7] - 4.0f * y * G[8];
  const float v3 = -4.0f * z * G[0] - 2.0f * w * G[1] + 2.0f * x * G[2] + 2.0f * w * G[3] -
                   4.0f * z * G[4] + 2.0f * y * G[5] + 2.0f * x * G[6] + 2.0f * y * G[7];
  const float v0 = -2.0f * z * G[1] + 2.0f * y * G[2] + 2.0f * z * G[3] - 2.0f * x * G[5] -
                   2.0f * y * G[6] + 2.0f * x * G[7];
  const float dot = v0 * w + v1 * x + v2 * y + v3 * z;
  vq[0] += (v0 - dot * w) * inv;
  vq[1] += (v1 - dot * x) * inv;
  vq[2] += (v2 - dot * y) * inv;
  vq[3] += (v3 - dot * z) * inv;
}

// gsplat_quat_scale_to_covar.cpp:278-333
__device__ __forceinline__ void qs_vjp(const float q[4], const float scale[3], const M3& r,
                                       const M3& vm, bool precision, float vq[4], float vs[3]) {
  float s[3] = {scale[0], scale[1], scale[2]};
  if (precision) {
    s[0] = 1.0f / s[0];
    s[1] = 1.0f / s[1];
    s[2] = 1.0f / s[2];
  }
  M3 m, v_m, v_r;
#pragma unroll
  for (int i = 0; i < 3; ++i)
#pragma unroll
    for (int j = 0; j < 3; ++j) m.v[i * 3 + j] = r.v[i * 3 + j] * s[j];
#pragma unroll
  for (int i = 0; i < 3; ++i)
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      float v = 0.0f;
#pragma unroll
      for (int k = 0; k < 3; ++k) v += (vm.v[i * 3 + k] + vm.v[k * 3 + i]) * m.v[k * 3 + j];
      v_m.v[i * 3 + j] = v;
      v_r.v[i * 3 + j] = v * s[j];
    }
  rotmat_vjp(q[0], q[1], q[2], q[3], v_r, vq);
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const float grad = r.v[j] * v_m.v[j] + r.v[3 + j] * v_m.v[3 + j] + r.v[6 + j] * v_m.v[6 + j];
    vs[j] += precision ? -s[j] * s[j] * grad : grad;
  }
}

__global__ void __launch_bounds__(256) qs2c_bwd_kernel(int64_t n, const float* __restrict__ quats,
                                                       const float* __restrict__ scales,
                                                       const float* __restrict__ v_covars,
                                                       const float* __restrict__ v_precis,
                                                       float* __restrict__ v_quats,
                                                       float* __restrict__ v_scales, int triu) {
  const int stride = triu ? 6 : 9;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n;
       e += (int64_t)gridDim.x * blockDim.x) {
    const float q[4] = {__ldg(quats + e * 4), __ldg(quats + e * 4 + 1), __ldg(quats + e * 4 + 2),
                        __ldg(quats + e * 4 + 3)};
    const float s[3] = {__ldg(scales + e * 3), __ldg(scales + e * 3 + 1),
                        __ldg(scales + e * 3 + 2)};
    const M3 r = rotmat(q[0], q[1], q[2], q[3]);
    float vq[4] = {0.f, 0.f, 0.f, 0.f}, vs[3] = {0.f, 0.f, 0.f};
    if (v_covars) qs_vjp(q, s, r, cot_matrix(triu, v_covars + e * stride), false, vq, vs);
    if (v_precis) qs_vjp(q, s, r, cot_matrix(triu, v_precis + e * stride), true, vq, vs);
#pragma unroll
    for (int a = 0; a < 4; ++a) v_quats[e * 4 + a] = vq[a];
#pragma unroll
    for (int a = 0; a < 3; ++a) v_scales[e * 3 + a] = vs[a];
  }
}

}  // namespace
}  // namespace gsb

extern "C" int gs_quat_scale_to_covar_fwd(const gs_qs2c_params* p, const float* quats,
                                          const float* scales, float* covars, float* precis,
                                          gs_stream_t stream) {
  using namespace gsb;
  if (!p || p->n < 0) return invalid("quat_scale_to_covar_fwd: bad params");
  if (p->n == 0) return GS_OK;
  if (!quats || !scales) return invalid("quat_scale_to_covar_fwd: quats and scales are required");
  if ((p->compute_covar && !covars) || (p->compute_preci && !precis))
    return invalid("quat_scale_to_covar_fwd: missing output buffer");
  qs2c_fwd_kernel<<<grid_for(p->n, 256), 256, 0, as_stream(stream)>>>(
      p->n, quats, scales, covars, precis, p->compute_covar, p->compute_preci, p->triu);
  return launch_status("quat_scale_to_covar_fwd");
}

extern "C" int gs_quat_scale_to_covar_bwd(const gs_qs2c_params* p, const float* quats,
                                          const float* scales, const float* v_covars,
                                          const float* v_precis, float* v_quats,
                                          float* v_scales, gs_stream_t stream) {
  using namespace gsb;
  if (!p || p->n < 0) return invalid("quat_scale_to_covar_bwd: bad params");
  if (p->n == 0) return GS_OK;
  if (!quats || !scales || !v_quats || !v_scales)
    return invalid("quat_scale_to_covar_bwd: missing buffer");
  if ((p->compute_covar && !v_covars) || (p->compute_preci && !v_precis))
    return invalid("quat_scale_to_covar_bwd: missing cotangent");
  qs2c_bwd_kernel<<<grid_for(p->n, 256), 256, 0, as_stream(stream)>>>(
      p->n, quats, scales, p->compute_covar ? v_covars : nullptr,
      p->compute_preci ? v_precis : nullptr, v_quats, v_scales, p->triu);
  return launch_status("quat_scale_to_covar_bwd");
}
