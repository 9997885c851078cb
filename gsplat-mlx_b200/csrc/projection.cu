// Fully fused EWA projection, forward and backward.
//
// Forward: one thread per (b, c, n) entry, grid-stride.  Arithmetic follows
// the reference CPU path operation by operation (gsplat_projection.cpp:
// 476-560) and this file is compiled without FMA contraction, so means2d,
// depths, conics and radii are bit-identical to the reference's eval_cpu --
// the depth bits become the low 32 bits of the intersection sort keys.
// Culling follows the Metal eval_gpu path that the Python binding runs
// (metal/gsplat_projection.metal:249-326): near/far, det <= 0, the opacity
// threshold, radius_clip with &&, and footprints entirely off the image.
// Camera models 1 (orthographic) and 2 (fisheye) follow metal:156-201.
//
// Backward: one thread per (b, n) Gaussian looping over its C cameras
// (metal:446-569), so per-Gaussian gradients need no atomics.  v_viewmats,
// when requested, is reduced over Gaussians per camera inside the same
// kernel (warp shuffle -> shared memory -> one atomicAdd per CTA and
// element), replacing the reference's O(N)-serial per-camera kernel
// (metal:571-676).
#include "common.cuh"

namespace gsb {
namespace {

constexpr float kAlphaThreshold = 1.0f / 255.0f;
constexpr float kGaussianExtend = 3.33f;
constexpr float kMinCompensation = 0.005f;

// ln x correctly rounded to float: CUDA's double logarithm (under one
// double ulp of error) rounded once.  The reference's std::log(float)
// (glibc logf) returns the same float on all but 0.2% of the floats in
// [1, 300] (exhaustive comparison), and there by one ulp; an integer
// radius moves only when extend * sqrt(cov) also lies within an ulp of an
// integer.  logf, by contrast, differs from it by up to an ulp on a large
// share of arguments.
__device__ __forceinline__ float log_cr(float x) { return __double2float_rn(log((double)x)); }

struct M3 {
  float v[9];
};

__device__ __forceinline__ M3 mul(const M3& a, const M3& b) {
  M3 o;
#pragma unroll
  for (int r = 0; r < 3; ++r)
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      float v = 0.0f;
#pragma unroll
      for (int k = 0; k < 3; ++k) v += a.v[r * 3 + k] * b.v[k * 3 + c];
      o.v[r * 3 + c] = v;
    }
  return o;
}

__device__ __forceinline__ M3 tr(const M3& a) {
  M3 o;
  o.v[0] = a.v[0]; o.v[1] = a.v[3]; o.v[2] = a.v[6];
  o.v[3] = a.v[1]; o.v[4] = a.v[4]; o.v[5] = a.v[7];
  o.v[6] = a.v[2]; o.v[7] = a.v[5]; o.v[8] = a.v[8];
  return o;
}

__device__ __forceinline__ M3 covar6(const float* c) {
  M3 o;
  o.v[0] = __ldg(c); o.v[1] = __ldg(c + 1); o.v[2] = __ldg(c + 2);
  o.v[3] = o.v[1];   o.v[4] = __ldg(c + 3); o.v[5] = __ldg(c + 4);
  o.v[6] = o.v[2];   o.v[7] = o.v[5];       o.v[8] = __ldg(c + 5);
  return o;
}

// gsplat_projection.cpp:182-206
__device__ __forceinline__ M3 quat_rot(const float q[4]) {
  float w = q[0], x = q[1], y = q[2], z = q[3];
  const float inv = 1.0f / sqrtf(w * w + x * x + y * y + z * z);
  w *= inv; x *= inv; y *= inv; z *= inv;
  const float x2 = x * x, y2 = y * y, z2 = z * z;
  const float xy = x * y, xz = x * z, yz = y * z;
  const float wx = w * x, wy = w * y, wz = w * z;
  M3 r;
  r.v[0] = 1.0f - 2.0f * (y2 + z2); r.v[1] = 2.0f * (xy - wz); r.v[2] = 2.0f * (xz + wy);
  r.v[3] = 2.0f * (xy + wz); r.v[4] = 1.0f - 2.0f * (x2 + z2); r.v[5] = 2.0f * (yz - wx);
  r.v[6] = 2.0f * (xz - wy); r.v[7] = 2.0f * (yz + wx); r.v[8] = 1.0f - 2.0f * (x2 + y2);
  return r;
}

// gsplat_projection.cpp:208-222: R diag(s)^2 R^T in the reference's order.
__device__ __forceinline__ M3 covar_qs(const float q[4], const float s[3]) {
  const M3 r = quat_rot(q);
  M3 o;
#pragma unroll
  for (int row = 0; row < 3; ++row)
#pragma unroll
    for (int col = 0; col < 3; ++col) {
      float v = 0.0f;
#pragma unroll
      for (int k = 0; k < 3; ++k) v += r.v[row * 3 + k] * s[k] * s[k] * r.v[col * 3 + k];
      o.v[row * 3 + col] = v;
    }
  return o;
}

struct Cam {
  M3 R;
  float t[3];
  float fx, fy, cx, cy;
};

__device__ __forceinline__ Cam load_cam(const float* view, const float* K) {
  Cam c;
  c.R.v[0] = __ldg(view + 0); c.R.v[1] = __ldg(view + 1); c.R.v[2] = __ldg(view + 2);
  c.R.v[3] = __ldg(view + 4); c.R.v[4] = __ldg(view + 5); c.R.v[5] = __ldg(view + 6);
  c.R.v[6] = __ldg(view + 8); c.R.v[7] = __ldg(view + 9); c.R.v[8] = __ldg(view + 10);
  c.t[0] = __ldg(view + 3); c.t[1] = __ldg(view + 7); c.t[2] = __ldg(view + 11);
  c.fx = __ldg(K + 0); c.fy = __ldg(K + 4); c.cx = __ldg(K + 2); c.cy = __ldg(K + 5);
  return c;
}

struct FwdArgs {
  int B, C, N, W, H;
  float eps2d, near_plane, far_plane, radius_clip;
  int calc_comp, camera_model, use_covars, use_opacities;
  int quats16;  // quats on a 16-byte boundary: read them as one float4
  const float *means, *covars, *quats, *scales, *opacities, *viewmats, *Ks;
  float *means2d, *depths, *conics, *comps;
  int32_t* radii;
};

__global__ void __launch_bounds__(256) proj_fwd_kernel(FwdArgs a) {
  const int64_t total = (int64_t)a.B * a.C * a.N;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t bc = idx / a.N;
    const int64_t n = idx - bc * a.N;
    const int64_t b = bc / a.C;
    const int64_t g = b * a.N + n;
    const Cam cam = load_cam(a.viewmats + bc * 16, a.Ks + bc * 9);
    const float mw[3] = {__ldg(a.means + g * 3), __ldg(a.means + g * 3 + 1),
                         __ldg(a.means + g * 3 + 2)};
    // quats / scales are read together with the means (before the near/far
    // test that may cull the entry), so their latency is not exposed twice
    float q[4] = {0.f, 0.f, 0.f, 0.f}, sc[3] = {0.f, 0.f, 0.f};
    if (!a.use_covars) {
      if (a.quats16) {
        const float4 q4 = __ldg(reinterpret_cast<const float4*>(a.quats) + g);
        q[0] = q4.x; q[1] = q4.y; q[2] = q4.z; q[3] = q4.w;
      } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) q[k] = __ldg(a.quats + g * 4 + k);
      }
      sc[0] = __ldg(a.scales + g * 3);
      sc[1] = __ldg(a.scales + g * 3 + 1);
      sc[2] = __ldg(a.scales + g * 3 + 2);
    }
    const M3& R = cam.R;
    const float mc0 = R.v[0] * mw[0] + R.v[1] * mw[1] + R.v[2] * mw[2] + cam.t[0];
    const float mc1 = R.v[3] * mw[0] + R.v[4] * mw[1] + R.v[5] * mw[2] + cam.t[1];
    const float mc2 = R.v[6] * mw[0] + R.v[7] * mw[1] + R.v[8] * mw[2] + cam.t[2];

    bool ok = !(mc2 < a.near_plane || mc2 > a.far_plane);
    float m2x = 0.f, m2y = 0.f, con0 = 0.f, con1 = 0.f, con2 = 0.f, comp = 0.f;
    int rxi = 0, ryi = 0;
    if (ok) {
      M3 cw;
      if (a.use_covars) {
        cw = covar6(a.covars + g * 6);
      } else {
        cw = covar_qs(q, sc);
      }
      const M3 cc = mul(mul(R, cw), tr(R));
      const float x = mc0, y = mc1, z = mc2;
      float J[6];
      if (a.camera_model == 1) {
        J[0] = cam.fx; J[1] = 0.0f; J[2] = 0.0f;
        J[3] = 0.0f; J[4] = cam.fy; J[5] = 0.0f;
        m2x = cam.fx * x + cam.cx;
        m2y = cam.fy * y + cam.cy;
      } else if (a.camera_model == 2) {
        const float eps = 0.0000001f;
        const float xy_len = sqrtf(x * x + y * y) + eps;
        const float theta = atan2f(xy_len, z + eps);
        m2x = x * cam.fx * theta / xy_len + cam.cx;
        m2y = y * cam.fy * theta / xy_len + cam.cy;
        const float x2 = x * x + eps, y2 = y * y, xy = x * y;
        const float x2y2 = x2 + y2;
        const float x2y2z2_inv = 1.0f / (x2y2 + z * z);
        const float bb = atan2f(xy_len, z) / xy_len / x2y2;
        const float aa = z * x2y2z2_inv / x2y2;
        J[0] = cam.fx * (x2 * aa + y2 * bb); J[1] = cam.fx * xy * (aa - bb);
        J[2] = -cam.fx * x * x2y2z2_inv;
        J[3] = cam.fy * xy * (aa - bb); J[4] = cam.fy * (y2 * aa + x2 * bb);
        J[5] = -cam.fy * y * x2y2z2_inv;
      } else {
        const float rz = 1.0f / z, rz2 = rz * rz;
        const float tan_fovx = 0.5f * (float)a.W / cam.fx;
        const float tan_fovy = 0.5f * (float)a.H / cam.fy;
        const float lim_x_pos = ((float)a.W - cam.cx) / cam.fx + 0.3f * tan_fovx;
        const float lim_x_neg = cam.cx / cam.fx + 0.3f * tan_fovx;
        const float lim_y_pos = ((float)a.H - cam.cy) / cam.fy + 0.3f * tan_fovy;
        const float lim_y_neg = cam.cy / cam.fy + 0.3f * tan_fovy;
        const float tx = z * fminf(lim_x_pos, fmaxf(-lim_x_neg, x * rz));
        const float ty = z * fminf(lim_y_pos, fmaxf(-lim_y_neg, y * rz));
        J[0] = cam.fx * rz; J[1] = 0.0f; J[2] = -cam.fx * tx * rz2;
        J[3] = 0.0f; J[4] = cam.fy * rz; J[5] = -cam.fy * ty * rz2;
        m2x = cam.fx * x * rz + cam.cx;
        m2y = cam.fy * y * rz + cam.cy;
      }
      float c2[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int i = 0; i < 3; ++i)
#pragma unroll
            for (int j = 0; j < 3; ++j) c2[r * 2 + c] += J[r * 3 + i] * cc.v[i * 3 + j] * J[c * 3 + j];
      const float det_orig = c2[0] * c2[3] - c2[1] * c2[2];
      c2[0] += a.eps2d;
      c2[3] += a.eps2d;
      const float det = c2[0] * c2[3] - c2[1] * c2[2];
      ok = det > 0.0f;
      if (ok) {
        const float inv_det = 1.0f / det;
        con0 = c2[3] * inv_det;
        con1 = -c2[1] * inv_det;
        con2 = c2[0] * inv_det;
        comp = sqrtf(fmaxf(kMinCompensation * kMinCompensation, det_orig / det));
        float extend = kGaussianExtend;
        if (a.use_opacities) {
          float op = __ldg(a.opacities + g);
          if (a.calc_comp) op *= comp;
          if (op < kAlphaThreshold) ok = false;
          else extend = fminf(kGaussianExtend, sqrtf(2.0f * log_cr(op / kAlphaThreshold)));
        }
        const float rx = ceilf(extend * sqrtf(c2[0]));
        const float ry = ceilf(extend * sqrtf(c2[3]));
        if (ok && rx <= a.radius_clip && ry <= a.radius_clip) ok = false;
        if (ok && (m2x + rx <= 0.0f || m2x - rx >= (float)a.W || m2y + ry <= 0.0f ||
                   m2y - ry >= (float)a.H))
          ok = false;
        rxi = (int)rx;
        ryi = (int)ry;
      }
    }
    if (!ok) {
      m2x = m2y = con0 = con1 = con2 = comp = 0.0f;
      rxi = ryi = 0;
    }
    a.radii[idx * 2] = rxi;
    a.radii[idx * 2 + 1] = ryi;
    a.means2d[idx * 2] = m2x;
    a.means2d[idx * 2 + 1] = m2y;
    a.depths[idx] = ok ? mc2 : 0.0f;
    a.conics[idx * 3] = con0;
    a.conics[idx * 3 + 1] = con1;
    a.conics[idx * 3 + 2] = con2;
    if (a.calc_comp) a.comps[idx] = comp;
  }
}

// ------------------------------------------------------------------ backward

struct BwdArgs {
  int B, C, N, W, H;
  float eps2d;
  int calc_comp, use_covars;
  const float *means, *covars, *quats, *scales, *viewmats, *Ks;
  const int32_t* radii;
  const float *conics, *comps, *v_means2d, *v_depths, *v_conics, *v_comps;
  float *v_means, *v_covars, *v_quats, *v_scales, *v_viewmats;
};

// gsplat_projection.cpp:298-376 (perspective projection VJP).
__device__ __forceinline__ void persp_vjp(const float mc[3], const M3& cc, const Cam& cam, int W,
                                          int H, const float vc2[4], float vm2x, float vm2y,
                                          float vmc[3], M3& vcc) {
  const float x = mc[0], y = mc[1], z = mc[2];
  const float fx = cam.fx, fy = cam.fy, cx = cam.cx, cy = cam.cy;
  const float tan_fovx = 0.5f * (float)W / fx;
  const float tan_fovy = 0.5f * (float)H / fy;
  const float lim_x_pos = ((float)W - cx) / fx + 0.3f * tan_fovx;
  const float lim_x_neg = cx / fx + 0.3f * tan_fovx;
  const float lim_y_pos = ((float)H - cy) / fy + 0.3f * tan_fovy;
  const float lim_y_neg = cy / fy + 0.3f * tan_fovy;
  const float rz = 1.0f / z, rz2 = rz * rz, rz3 = rz2 * rz;
  const float x_rz = x * rz, y_rz = y * rz;
  const float tx = z * fminf(lim_x_pos, fmaxf(-lim_x_neg, x_rz));
  const float ty = z * fminf(lim_y_pos, fmaxf(-lim_y_neg, y_rz));
  const float J[6] = {fx * rz, 0.0f, -fx * tx * rz2, 0.0f, fy * rz, -fy * ty * rz2};
#pragma unroll
  for (int i = 0; i < 3; ++i)
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      float v = 0.0f;
#pragma unroll
      for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int c = 0; c < 2; ++c) v += J[r * 3 + i] * vc2[r * 2 + c] * J[c * 3 + j];
      vcc.v[i * 3 + j] = v;
    }
  vmc[0] += fx * rz * vm2x;
  vmc[1] += fy * rz * vm2y;
  vmc[2] += -(fx * x * vm2x + fy * y * vm2y) * rz2;
  float vJ[6];
#pragma unroll
  for (int r = 0; r < 2; ++r)
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      float left = 0.0f, right = 0.0f;
#pragma unroll
      for (int c = 0; c < 2; ++c)
#pragma unroll
        for (int j = 0; j < 3; ++j) {
          left += vc2[r * 2 + c] * J[c * 3 + j] * cc.v[i * 3 + j];
          right += vc2[c * 2 + r] * J[c * 3 + j] * cc.v[j * 3 + i];
        }
      vJ[r * 3 + i] = left + right;
    }
  if (x_rz <= lim_x_pos && x_rz >= -lim_x_neg) vmc[0] += -fx * rz2 * vJ[2];
  else vmc[2] += -fx * rz3 * tx * vJ[2];
  if (y_rz <= lim_y_pos && y_rz >= -lim_y_neg) vmc[1] += -fy * rz2 * vJ[5];
  else vmc[2] += -fy * rz3 * ty * vJ[5];
  vmc[2] += -fx * rz2 * vJ[0] - fy * rz2 * vJ[4] + 2.0f * fx * tx * rz3 * vJ[2] +
            2.0f * fy * ty * rz3 * vJ[5];
}

// gsplat_projection.cpp:410-474: VJP of R(q) diag(s)^2 R(q)^T.
__device__ __forceinline__ void qs_covar_vjp(const float q[4], const float s[3], const M3& vcw,
                                             float vq[4], float vs[3]) {
  const M3 R = quat_rot(q);
  M3 M, sym;
#pragma unroll
  for (int r = 0; r < 3; ++r)
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      M.v[r * 3 + c] = R.v[r * 3 + c] * s[c];
      sym.v[r * 3 + c] = vcw.v[r * 3 + c] + vcw.v[c * 3 + r];
    }
  const M3 vM = mul(sym, M);
  M3 vR;
#pragma unroll
  for (int r = 0; r < 3; ++r)
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      vR.v[r * 3 + c] = vM.v[r * 3 + c] * s[c];
      vs[c] += vM.v[r * 3 + c] * R.v[r * 3 + c];
    }
  float w = q[0], x = q[1], y = q[2], z = q[3];
  const float inv = 1.0f / sqrtf(w * w + x * x + y * y + z * z);
  w *= inv; x *= inv; y *= inv; z *= inv;
  const float* g = vR.v;
  const float vn[4] = {
      2.0f * (x * (g[7] - g[5]) + y * (g[2] - g[6]) + z * (g[3] - g[1])),
      2.0f * (-2.0f * x * (g[4] + g[8]) + y * (g[1] + g[3]) + z * (g[2] + g[6]) + w * (g[7] - g[5])),
      2.0f * (x * (g[1] + g[3]) - 2.0f * y * (g[0] + g[8]) + z * (g[5] + g[7]) + w * (g[2] - g[6])),
      2.0f * (x * (g[2] + g[6]) + y * (g[5] + g[7]) - 2.0f * z * (g[0] + g[4]) + w * (g[3] - g[1]))};
  const float dot = vn[0] * w + vn[1] * x + vn[2] * y + vn[3] * z;
  vq[0] += (vn[0] - dot * w) * inv;
  vq[1] += (vn[1] - dot * x) * inv;
  vq[2] += (vn[2] - dot * y) * inv;
  vq[3] += (vn[3] - dot * z) * inv;
}

// Gradient terms of one visible (camera, Gaussian) entry: adds the
// world-mean and world-covariance VJPs of the projection to vmw and vcw_tot
// and, with want_view, writes the entry's 12 view-matrix terms to vR.
__device__ __forceinline__ void entry_vjp(const BwdArgs& a, int64_t bc, int64_t idx,
                                          const float mw[3], const M3& cw, bool want_view,
                                          float vmw[3], M3& vcw_tot, float vR[12]) {
    const Cam cam = load_cam(a.viewmats + bc * 16, a.Ks + bc * 9);
    const float ci[4] = {__ldg(a.conics + idx * 3), __ldg(a.conics + idx * 3 + 1),
                         __ldg(a.conics + idx * 3 + 1), __ldg(a.conics + idx * 3 + 2)};
    const float vco1 = 0.5f * __ldg(a.v_conics + idx * 3 + 1);
    const float vci[4] = {__ldg(a.v_conics + idx * 3), vco1, vco1, __ldg(a.v_conics + idx * 3 + 2)};
    const float t0[4] = {ci[0] * vci[0] + ci[1] * vci[2], ci[0] * vci[1] + ci[1] * vci[3],
                         ci[2] * vci[0] + ci[3] * vci[2], ci[2] * vci[1] + ci[3] * vci[3]};
    float vc2[4] = {-(t0[0] * ci[0] + t0[1] * ci[2]), -(t0[0] * ci[1] + t0[1] * ci[3]),
                    -(t0[2] * ci[0] + t0[3] * ci[2]), -(t0[2] * ci[1] + t0[3] * ci[3])};
    if (a.calc_comp && a.v_comps) {
      // gsplat_projection.cpp:277-296
      const float comp = __ldg(a.comps + idx);
      const float det = ci[0] * ci[3] - ci[1] * ci[2];
      const float v_sqr = __ldg(a.v_comps + idx) * 0.5f / (comp + 1.0e-6f);
      const float om = 1.0f - comp * comp;
      vc2[0] += v_sqr * (om * ci[0] - a.eps2d * det);
      vc2[1] += v_sqr * (om * ci[1]);
      vc2[2] += v_sqr * (om * ci[2]);
      vc2[3] += v_sqr * (om * ci[3] - a.eps2d * det);
    }
    const M3& R = cam.R;
    const float mc[3] = {R.v[0] * mw[0] + R.v[1] * mw[1] + R.v[2] * mw[2] + cam.t[0],
                         R.v[3] * mw[0] + R.v[4] * mw[1] + R.v[5] * mw[2] + cam.t[1],
                         R.v[6] * mw[0] + R.v[7] * mw[1] + R.v[8] * mw[2] + cam.t[2]};
    const M3 cc = mul(mul(R, cw), tr(R));
    float vmc[3] = {0.0f, 0.0f, __ldg(a.v_depths + idx)};
    M3 vcc;
    persp_vjp(mc, cc, cam, a.W, a.H, vc2, __ldg(a.v_means2d + idx * 2),
              __ldg(a.v_means2d + idx * 2 + 1), vmc, vcc);
    // pos_w2c_vjp / covar_w2c_vjp, gsplat_projection.cpp:378-408
    vmw[0] += R.v[0] * vmc[0] + R.v[3] * vmc[1] + R.v[6] * vmc[2];
    vmw[1] += R.v[1] * vmc[0] + R.v[4] * vmc[1] + R.v[7] * vmc[2];
    vmw[2] += R.v[2] * vmc[0] + R.v[5] * vmc[1] + R.v[8] * vmc[2];
    const M3 Rt = tr(R);
    const M3 vcw = mul(mul(Rt, vcc), R);
#pragma unroll
    for (int i = 0; i < 9; ++i) vcw_tot.v[i] += vcw.v[i];
    if (want_view) {
      const M3 term1 = mul(mul(vcc, R), tr(cw));
      const M3 term2 = mul(mul(tr(vcc), R), cw);
#pragma unroll
      for (int r = 0; r < 3; ++r) {
#pragma unroll
        for (int cc2 = 0; cc2 < 3; ++cc2)
          vR[r * 3 + cc2] = vmc[r] * mw[cc2] + term1.v[r * 3 + cc2] + term2.v[r * 3 + cc2];
        vR[9 + r] = vmc[r];
      }
    }
}

// A Gaussian's world mean and covariance (given, or from quats and scales).
__device__ __forceinline__ void load_gauss(const BwdArgs& a, int64_t g, float mw[3], float q[4],
                                           float s[3], M3& cw) {
  mw[0] = __ldg(a.means + g * 3);
  mw[1] = __ldg(a.means + g * 3 + 1);
  mw[2] = __ldg(a.means + g * 3 + 2);
  if (a.use_covars) {
    cw = covar6(a.covars + g * 6);
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) q[i] = __ldg(a.quats + g * 4 + i);
#pragma unroll
    for (int i = 0; i < 3; ++i) s[i] = __ldg(a.scales + g * 3 + i);
    cw = covar_qs(q, s);
  }
}

// A Gaussian's gradients, summed over its cameras: v_means and v_covars, or
// v_quats and v_scales through the covariance VJP.
__device__ __forceinline__ void store_gauss(const BwdArgs& a, int64_t g, const float q[4],
                                            const float s[3], const float vmw[3],
                                            const M3& vcw_tot) {
  a.v_means[g * 3] = vmw[0];
  a.v_means[g * 3 + 1] = vmw[1];
  a.v_means[g * 3 + 2] = vmw[2];
  if (a.use_covars) {
    float* o = a.v_covars + g * 6;
    o[0] = vcw_tot.v[0];
    o[1] = vcw_tot.v[1] + vcw_tot.v[3];
    o[2] = vcw_tot.v[2] + vcw_tot.v[6];
    o[3] = vcw_tot.v[4];
    o[4] = vcw_tot.v[5] + vcw_tot.v[7];
    o[5] = vcw_tot.v[8];
  } else {
    float vq[4] = {0.f, 0.f, 0.f, 0.f}, vs[3] = {0.f, 0.f, 0.f};
    qs_covar_vjp(q, s, vcw_tot, vq, vs);
#pragma unroll
    for (int i = 0; i < 4; ++i) a.v_quats[g * 4 + i] = vq[i];
#pragma unroll
    for (int i = 0; i < 3; ++i) a.v_scales[g * 3 + i] = vs[i];
  }
}

// Dynamic shared memory: per-camera v_viewmats partial sums [C][12].
__global__ void __launch_bounds__(256) proj_bwd_kernel(BwdArgs a, int smem_cams) {
  extern __shared__ float s_vview[];
  const bool want_view = a.v_viewmats != nullptr;
  const bool use_smem = want_view && smem_cams > 0;
  if (use_smem) {
    for (int i = threadIdx.x; i < a.C * 12; i += blockDim.x) s_vview[i] = 0.0f;
    __syncthreads();
  }
  const int64_t total = (int64_t)a.B * a.N;
  // Every thread of the CTA runs the same number of outer iterations so
  // that the per-camera warp reductions see full warps.
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t iters = (total + stride - 1) / stride;
  const int lane = threadIdx.x & 31;
  for (int64_t it = 0; it < iters; ++it) {
    const int64_t gidx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x + it * stride;
    const bool live = gidx < total;
    const int64_t b = live ? gidx / a.N : 0;
    const int64_t n = live ? gidx - b * a.N : 0;
    const int64_t g = b * a.N + n;
    float mw[3] = {0.f, 0.f, 0.f}, q[4] = {1.f, 0.f, 0.f, 0.f}, s[3] = {1.f, 1.f, 1.f};
    M3 cw = {};
    if (live) load_gauss(a, g, mw, q, s, cw);
    float vmw[3] = {0.f, 0.f, 0.f};
    M3 vcw_tot = {};
    for (int c = 0; c < a.C; ++c) {
      const int64_t bc = b * a.C + c;
      const int64_t idx = bc * a.N + n;
      bool act = live && __ldg(a.radii + idx * 2) > 0 && __ldg(a.radii + idx * 2 + 1) > 0;
      float vR[12];
#pragma unroll
      for (int i = 0; i < 12; ++i) vR[i] = 0.0f;
      if (act) entry_vjp(a, bc, idx, mw, cw, want_view, vmw, vcw_tot, vR);
      if (want_view && a.B > 1) {
        // Lanes of one warp may belong to different batches: no warp sum.
        if (act) {
#pragma unroll
          for (int i = 0; i < 12; ++i) {
            const int r = i < 9 ? i / 3 : i - 9;
            const int col = i < 9 ? i % 3 : 3;
            atomicAdd(a.v_viewmats + bc * 16 + r * 4 + col, vR[i]);
          }
        }
      } else if (want_view) {
        // B == 1: reduce the 12 v_viewmats terms of this camera over the
        // warp, then over the CTA in shared memory (or straight to global).
        const bool any = __any_sync(0xffffffffu, act);
        if (any) {
#pragma unroll
          for (int i = 0; i < 12; ++i) vR[i] = warp_sum(vR[i]);
          if (lane == 0) {
            float* dst = use_smem ? s_vview + c * 12 : nullptr;
#pragma unroll
            for (int i = 0; i < 12; ++i) {
              if (use_smem) {
                atomicAdd(dst + i, vR[i]);
              } else {
                const int r = i < 9 ? i / 3 : i - 9;
                const int col = i < 9 ? i % 3 : 3;
                atomicAdd(a.v_viewmats + bc * 16 + r * 4 + col, vR[i]);
              }
            }
          }
        }
      }
    }
    if (live) store_gauss(a, g, q, s, vmw, vcw_tot);
  }
  if (use_smem) {
    __syncthreads();
    // Only batch 0 of B is handled through shared memory (smem_cams == C
    // requires B == 1); see the launch below.
    for (int i = threadIdx.x; i < a.C * 12; i += blockDim.x) {
      const int c = i / 12, k = i % 12;
      const int r = k < 9 ? k / 3 : k - 9;
      const int col = k < 9 ? k % 3 : 3;
      const float v = s_vview[i];
      if (v != 0.0f) atomicAdd(a.v_viewmats + (int64_t)c * 16 + r * 4 + col, v);
    }
  }
}

// The form without v_viewmats (the training step's): each warp walks chunks
// of 32 Gaussians; those no camera sees get zero gradients at once, the
// others go to a per-warp queue in shared memory and are processed 32 at a
// time, one per lane, so that the per-camera VJPs and the covariance VJP run
// on full warps (about a third of the Gaussians are visible in a training
// view).  Same arithmetic per Gaussian as proj_bwd_kernel.
constexpr int kProjBwdWarps = 4;

__device__ __forceinline__ void proj_bwd_one(const BwdArgs& a, int64_t g) {
  const int64_t b = g / a.N, n = g - b * a.N;
  float mw[3], q[4] = {1.f, 0.f, 0.f, 0.f}, s[3] = {1.f, 1.f, 1.f};
  M3 cw;
  load_gauss(a, g, mw, q, s, cw);
  float vmw[3] = {0.f, 0.f, 0.f};
  M3 vcw_tot = {};
  float vR[12];
  for (int c = 0; c < a.C; ++c) {
    const int64_t bc = b * a.C + c;
    const int64_t idx = bc * a.N + n;
    if (__ldg(a.radii + idx * 2) > 0 && __ldg(a.radii + idx * 2 + 1) > 0)
      entry_vjp(a, bc, idx, mw, cw, false, vmw, vcw_tot, vR);
  }
  store_gauss(a, g, q, s, vmw, vcw_tot);
}

__global__ void __launch_bounds__(32 * kProjBwdWarps) proj_bwd_queue_kernel(BwdArgs a) {
  __shared__ int64_t s_q[kProjBwdWarps][64];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int64_t* qu = s_q[warp];
  int qn = 0;  // queued entries, < 32 between chunks
  const int64_t total = (int64_t)a.B * a.N;
  const int64_t chunks = (total + 31) / 32;
  for (int64_t ch = (int64_t)blockIdx.x * kProjBwdWarps + warp; ch < chunks;
       ch += (int64_t)gridDim.x * kProjBwdWarps) {
    const int64_t g = ch * 32 + lane;
    bool any = false;
    if (g < total) {
      const int64_t b = g / a.N, n = g - b * a.N;
      for (int c = 0; c < a.C; ++c) {
        const int64_t idx = (b * a.C + c) * a.N + n;
        any |= __ldg(a.radii + idx * 2) > 0 && __ldg(a.radii + idx * 2 + 1) > 0;
      }
      if (!any) {  // no camera sees it: every gradient is zero
        a.v_means[g * 3] = a.v_means[g * 3 + 1] = a.v_means[g * 3 + 2] = 0.0f;
        if (a.use_covars) {
#pragma unroll
          for (int i = 0; i < 6; ++i) a.v_covars[g * 6 + i] = 0.0f;
        } else {
#pragma unroll
          for (int i = 0; i < 4; ++i) a.v_quats[g * 4 + i] = 0.0f;
#pragma unroll
          for (int i = 0; i < 3; ++i) a.v_scales[g * 3 + i] = 0.0f;
        }
      }
    }
    const unsigned bal = __ballot_sync(0xffffffffu, any);
    if (any) qu[qn + __popc(bal & ((1u << lane) - 1u))] = g;
    qn += __popc(bal);
    __syncwarp();
    if (qn >= 32) {
      proj_bwd_one(a, qu[qn - 32 + lane]);
      qn -= 32;
      __syncwarp();
    }
  }
  if (lane < qn) proj_bwd_one(a, qu[lane]);
}

}  // namespace
}  // namespace gsb

extern "C" int gs_projection_fwd(const gs_projection_params* p, const float* means,
                                 const float* covars, const float* quats, const float* scales,
                                 const float* opacities, const float* viewmats, const float* Ks,
                                 float* means2d, float* depths, float* conics,
                                 float* compensations, int32_t* radii, gs_stream_t stream) {
  using namespace gsb;
  if (!p || p->B < 0 || p->C < 0 || p->N < 0) return invalid("projection_fwd: bad params");
  const int64_t total = (int64_t)p->B * p->C * p->N;
  if (total == 0) return GS_OK;
  if (!means || !viewmats || !Ks || !means2d || !depths || !conics || !radii)
    return invalid("projection_fwd: missing buffer");
  if (p->use_covars ? !covars : (!quats || !scales))
    return invalid("projection_ewa_3dgs_fused_forward expects covars or quats+scales.");
  if (p->use_opacities && !opacities) return invalid("projection_fwd: opacities missing");
  if (p->calc_compensations && !compensations)
    return invalid("projection_fwd: compensations buffer missing");
  if (p->camera_model < 0 || p->camera_model > 2) return invalid("projection_fwd: camera_model");
  FwdArgs a{p->B, p->C, p->N, p->image_width, p->image_height, p->eps2d, p->near_plane,
            p->far_plane, p->radius_clip, p->calc_compensations, p->camera_model,
            p->use_covars, p->use_opacities,
            (int)((reinterpret_cast<uintptr_t>(quats) & 15) == 0), means, covars, quats, scales,
            opacities, viewmats, Ks, means2d, depths, conics, compensations, radii};
  proj_fwd_kernel<<<grid_for(total, 256), 256, 0, as_stream(stream)>>>(a);
  return launch_status("projection_fwd");
}

extern "C" int gs_projection_bwd(const gs_projection_params* p, const float* means,
                                 const float* covars, const float* quats, const float* scales,
                                 const float* viewmats, const float* Ks, const int32_t* radii,
                                 const float* conics, const float* compensations,
                                 const float* v_means2d, const float* v_depths,
                                 const float* v_conics, const float* v_compensations,
                                 float* v_means, float* v_covars, float* v_quats,
                                 float* v_scales, float* v_viewmats, gs_stream_t stream) {
  using namespace gsb;
  if (!p || p->B < 0 || p->C < 0 || p->N < 0) return invalid("projection_bwd: bad params");
  if (p->camera_model != 0)
    return invalid("projection_ewa_3dgs_fused_backward currently supports pinhole only.");
  cudaStream_t s = as_stream(stream);
  if (v_viewmats && (int64_t)p->B * p->C > 0) {
    if (cudaMemsetAsync(v_viewmats, 0, sizeof(float) * 16 * (size_t)p->B * p->C, s) != cudaSuccess)
      return launch_status("projection_bwd: memset v_viewmats");
  }
  const int64_t total = (int64_t)p->B * p->N;
  if (total == 0) return GS_OK;
  if (!means || !viewmats || !Ks || !radii || !conics || !v_means2d || !v_depths || !v_conics ||
      !v_means)
    return invalid("projection_bwd: missing buffer");
  if (p->use_covars ? (!covars || !v_covars) : (!quats || !scales || !v_quats || !v_scales))
    return invalid("projection_bwd: missing covariance buffers");
  if (p->calc_compensations && v_compensations && !compensations)
    return invalid("projection_bwd: compensations missing");
  BwdArgs a{p->B, p->C, p->N, p->image_width, p->image_height, p->eps2d,
            p->calc_compensations, p->use_covars, means, covars, quats, scales, viewmats, Ks,
            radii, conics, compensations, v_means2d, v_depths, v_conics,
            p->calc_compensations ? v_compensations : nullptr, v_means, v_covars, v_quats,
            v_scales, v_viewmats};
  // v_viewmats partial sums live in shared memory when they fit and B == 1.
  int smem_cams = (v_viewmats && p->B == 1 && p->C <= 1024) ? p->C : 0;
  const size_t smem = sizeof(float) * 12 * (size_t)smem_cams;
  if (smem > 48 * 1024) {
    cudaFuncSetAttribute(proj_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  }
  if (!v_viewmats) {
    proj_bwd_queue_kernel<<<grid_for(ceil_div(total, 32), kProjBwdWarps, 4),
                            32 * kProjBwdWarps, 0, s>>>(a);
    return launch_status("projection_bwd");
  }
  proj_bwd_kernel<<<grid_for(total, 256, 4), 256, smem, s>>>(a, smem_cams);
  return launch_status("projection_bwd");
}
