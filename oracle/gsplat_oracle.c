/*
 * CPU oracle: plain-C restatement of gsplat-mlx's gsplat_core CPU algorithms.
 * TEST INFRASTRUCTURE ONLY (see gsplat_oracle.h).  Each function cites the
 * reference file:line it restates.  Arithmetic is kept in the reference's
 * order so that float results agree closely; integer results (radii, tile
 * counts, keys, sort order, offsets, last ids) must agree exactly.
 *
 * Known difference from the reference CPU path, on purpose: the projection
 * forward applies the Metal eval_gpu culling (radius_clip with && and the
 * off-screen footprint test, gsplat_core/metal/gsplat_projection.metal:
 * 314-326) and its orthographic / fisheye models (:156-201), because the
 * Python binding runs eval_gpu (binding/binding.cpp:93).
 */
#include "gsplat_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

#define ORC_ERR_ARG (-1)
#define ORC_ERR_VALUE (-2)
#define ORC_ERR_OOB (-3)
#define ORC_ERR_NOMEM (-4)

/* ------------------------------------------------------------------ */
/* quaternion / covariance helpers                                     */
/* ------------------------------------------------------------------ */

/* gsplat_quat_scale_to_covar.cpp:103-138 (throws on a zero quaternion). */
static int qs_rotmat(const float* q, float r[9]) {
  float w = q[0], x = q[1], y = q[2], z = q[3];
  const float norm = sqrtf(w * w + x * x + y * y + z * z);
  if (norm == 0.0f) return ORC_ERR_VALUE;
  w /= norm;
  x /= norm;
  y /= norm;
  z /= norm;
  const float x2 = x * x, y2 = y * y, z2 = z * z;
  const float xy = x * y, xz = x * z, yz = y * z;
  const float wx = w * x, wy = w * y, wz = w * z;
  r[0] = 1.0f - 2.0f * (y2 + z2);
  r[1] = 2.0f * (xy - wz);
  r[2] = 2.0f * (xz + wy);
  r[3] = 2.0f * (xy + wz);
  r[4] = 1.0f - 2.0f * (x2 + z2);
  r[5] = 2.0f * (yz - wx);
  r[6] = 2.0f * (xz - wy);
  r[7] = 2.0f * (yz + wx);
  r[8] = 1.0f - 2.0f * (x2 + y2);
  return 0;
}

/* gsplat_quat_scale_to_covar.cpp:140-164: R diag(s^2) R^T, or with 1/s. */
static int qs_matrix(const float r[9], const float* scale, int precision,
                     float out[9]) {
  float s[3] = {scale[0], scale[1], scale[2]};
  if (precision) {
    if (s[0] == 0.0f || s[1] == 0.0f || s[2] == 0.0f) return ORC_ERR_VALUE;
    s[0] = 1.0f / s[0];
    s[1] = 1.0f / s[1];
    s[2] = 1.0f / s[2];
  }
  for (int row = 0; row < 3; ++row) {
    for (int col = 0; col < 3; ++col) {
      float v = 0.0f;
      for (int k = 0; k < 3; ++k) v += r[row * 3 + k] * s[k] * s[k] * r[col * 3 + k];
      out[row * 3 + col] = v;
    }
  }
  return 0;
}

/* gsplat_quat_scale_to_covar.cpp:166-179 */
static void qs_write(const float m[9], int triu, float* out) {
  if (triu) {
    out[0] = m[0];
    out[1] = m[1];
    out[2] = m[2];
    out[3] = m[4];
    out[4] = m[5];
    out[5] = m[8];
  } else {
    for (int i = 0; i < 9; ++i) out[i] = m[i];
  }
}

/* gsplat_quat_scale_to_covar.cpp:215-236: symmetric split of a triu cotangent. */
static void qs_cot_matrix(int triu, const float* cot, float out[9]) {
  if (triu) {
    out[0] = cot[0];
    out[1] = 0.5f * cot[1];
    out[2] = 0.5f * cot[2];
    out[3] = 0.5f * cot[1];
    out[4] = cot[3];
    out[5] = 0.5f * cot[4];
    out[6] = 0.5f * cot[2];
    out[7] = 0.5f * cot[4];
    out[8] = cot[5];
  } else {
    for (int i = 0; i < 9; ++i) out[i] = cot[i];
  }
}

/* gsplat_quat_scale_to_covar.cpp:238-276 */
static int qs_rotmat_vjp(const float* q, const float g[9], float* v_quat) {
  float w = q[0], x = q[1], y = q[2], z = q[3];
  const float norm = sqrtf(w * w + x * x + y * y + z * z);
  if (norm == 0.0f) return ORC_ERR_VALUE;
  const float inv = 1.0f / norm;
  w *= inv;
  x *= inv;
  y *= inv;
  z *= inv;
  float vn[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  vn[1] += 2.0f * y * g[1] + 2.0f * z * g[2] + 2.0f * y * g[3] -
           4.0f * x * g[4] - 2.0f * w * g[5] + 2.0f * z * g[6] +
           2.0f * w * g[7] - 4.0f * x * g[8];
  vn[2] += -4.0f * y * g[0] + 2.0f * x * g[1] + 2.0f * w * g[2] +
           2.0f * x * g[3] + 2.0f * z * g[5] - 2.0f * w * g[6] +
           2.0f * z * g[7] - 4.0f * y * g[8];
  vn[3] += -4.0f * z * g[0] - 2.0f * w * g[1] + 2.0f * x * g[2] +
           2.0f * w * g[3] - 4.0f * z * g[4] + 2.0f * y * g[5] +
           2.0f * x * g[6] + 2.0f * y * g[7];
  vn[0] += -2.0f * z * g[1] + 2.0f * y * g[2] + 2.0f * z * g[3] -
           2.0f * x * g[5] - 2.0f * y * g[6] + 2.0f * x * g[7];
  const float dot = vn[0] * w + vn[1] * x + vn[2] * y + vn[3] * z;
  v_quat[0] += (vn[0] - dot * w) * inv;
  v_quat[1] += (vn[1] - dot * x) * inv;
  v_quat[2] += (vn[2] - dot * y) * inv;
  v_quat[3] += (vn[3] - dot * z) * inv;
  return 0;
}

/* gsplat_quat_scale_to_covar.cpp:278-333 */
static int qs_vjp(const float* q, const float* scale, const float r[9],
                  const float vm[9], int precision, float* v_quat,
                  float* v_scale) {
  float s[3] = {scale[0], scale[1], scale[2]};
  if (precision) {
    if (s[0] == 0.0f || s[1] == 0.0f || s[2] == 0.0f) return ORC_ERR_VALUE;
    s[0] = 1.0f / s[0];
    s[1] = 1.0f / s[1];
    s[2] = 1.0f / s[2];
  }
  float m[9], v_m[9], v_r[9];
  for (int row = 0; row < 3; ++row)
    for (int col = 0; col < 3; ++col) m[row * 3 + col] = r[row * 3 + col] * s[col];
  for (int row = 0; row < 3; ++row) {
    for (int col = 0; col < 3; ++col) {
      float v = 0.0f;
      for (int k = 0; k < 3; ++k)
        v += (vm[row * 3 + k] + vm[k * 3 + row]) * m[k * 3 + col];
      v_m[row * 3 + col] = v;
    }
  }
  for (int row = 0; row < 3; ++row)
    for (int col = 0; col < 3; ++col) v_r[row * 3 + col] = v_m[row * 3 + col] * s[col];
  int rc = qs_rotmat_vjp(q, v_r, v_quat);
  if (rc) return rc;
  for (int col = 0; col < 3; ++col) {
    float grad = 0.0f;
    for (int row = 0; row < 3; ++row) grad += r[row * 3 + col] * v_m[row * 3 + col];
    if (precision) {
      v_scale[col] += -s[col] * s[col] * grad;
    } else {
      v_scale[col] += grad;
    }
  }
  return 0;
}

/* gsplat_quat_scale_to_covar.cpp:374-405 */
int orc_qs2c_fwd(int64_t n, const float* quats, const float* scales,
                 int compute_covar, int compute_preci, int triu, float* covars,
                 float* precis) {
  if (n < 0) return ORC_ERR_ARG;
  const int stride = triu ? 6 : 9;
  for (int64_t e = 0; e < n; ++e) {
    float r[9], m[9];
    int rc = qs_rotmat(quats + e * 4, r);
    if (rc) return rc;
    if (compute_covar) {
      qs_matrix(r, scales + e * 3, 0, m);
      qs_write(m, triu, covars + e * stride);
    }
    if (compute_preci) {
      rc = qs_matrix(r, scales + e * 3, 1, m);
      if (rc) return rc;
      qs_write(m, triu, precis + e * stride);
    }
  }
  return 0;
}

/* gsplat_quat_scale_to_covar.cpp:407-468 */
int orc_qs2c_bwd(int64_t n, const float* quats, const float* scales,
                 const float* v_covars, const float* v_precis, int triu,
                 float* v_quats, float* v_scales) {
  if (n < 0) return ORC_ERR_ARG;
  const int stride = triu ? 6 : 9;
  for (int64_t e = 0; e < n; ++e) {
    float vq[4] = {0, 0, 0, 0}, vs[3] = {0, 0, 0};
    float r[9], cm[9];
    int rc = qs_rotmat(quats + e * 4, r);
    if (rc) return rc;
    if (v_covars) {
      qs_cot_matrix(triu, v_covars + e * stride, cm);
      rc = qs_vjp(quats + e * 4, scales + e * 3, r, cm, 0, vq, vs);
      if (rc) return rc;
    }
    if (v_precis) {
      qs_cot_matrix(triu, v_precis + e * stride, cm);
      rc = qs_vjp(quats + e * 4, scales + e * 3, r, cm, 1, vq, vs);
      if (rc) return rc;
    }
    for (int a = 0; a < 4; ++a) v_quats[e * 4 + a] = vq[a];
    for (int a = 0; a < 3; ++a) v_scales[e * 3 + a] = vs[a];
  }
  return 0;
}

/* ------------------------------------------------------------------ */
/* projection                                                          */
/* ------------------------------------------------------------------ */

static void m3_mul(const float a[9], const float b[9], float o[9]) {
  for (int r = 0; r < 3; ++r)
    for (int c = 0; c < 3; ++c) {
      float v = 0.0f;
      for (int k = 0; k < 3; ++k) v += a[r * 3 + k] * b[k * 3 + c];
      o[r * 3 + c] = v;
    }
}

static void m3_t(const float a[9], float o[9]) {
  o[0] = a[0]; o[1] = a[3]; o[2] = a[6];
  o[3] = a[1]; o[4] = a[4]; o[5] = a[7];
  o[6] = a[2]; o[7] = a[5]; o[8] = a[8];
}

/* gsplat_projection.cpp:174-180 */
static void read_covar6(const float* c, float o[9]) {
  o[0] = c[0]; o[1] = c[1]; o[2] = c[2];
  o[3] = c[1]; o[4] = c[3]; o[5] = c[4];
  o[6] = c[2]; o[7] = c[4]; o[8] = c[5];
}

/* gsplat_projection.cpp:182-222 (1/sqrt normalisation, no zero check). */
static void proj_covar_from_qs(const float* q, const float* s, float o[9]) {
  float w = q[0], x = q[1], y = q[2], z = q[3];
  const float inv = 1.0f / sqrtf(w * w + x * x + y * y + z * z);
  w *= inv; x *= inv; y *= inv; z *= inv;
  const float x2 = x * x, y2 = y * y, z2 = z * z;
  const float xy = x * y, xz = x * z, yz = y * z;
  const float wx = w * x, wy = w * y, wz = w * z;
  const float r[9] = {1.0f - 2.0f * (y2 + z2), 2.0f * (xy - wz), 2.0f * (xz + wy),
                      2.0f * (xy + wz), 1.0f - 2.0f * (x2 + z2), 2.0f * (yz - wx),
                      2.0f * (xz - wy), 2.0f * (yz + wx), 1.0f - 2.0f * (x2 + y2)};
  for (int row = 0; row < 3; ++row)
    for (int col = 0; col < 3; ++col) {
      float v = 0.0f;
      for (int k = 0; k < 3; ++k) v += r[row * 3 + k] * s[k] * s[k] * r[col * 3 + k];
      o[row * 3 + col] = v;
    }
}

static void view_rt(const float* v, float R[9], float t[3]) {
  R[0] = v[0]; R[1] = v[1]; R[2] = v[2];
  R[3] = v[4]; R[4] = v[5]; R[5] = v[6];
  R[6] = v[8]; R[7] = v[9]; R[8] = v[10];
  t[0] = v[3]; t[1] = v[7]; t[2] = v[11];
}

/*
 * One (camera, Gaussian) forward: gsplat_projection.cpp:476-560 for the
 * pinhole math, metal/gsplat_projection.metal:156-201 for the other models.
 * Returns 1 when the entry survives the near/far and determinant tests.
 */
static int proj_eval(const float* mean_w, const float* covar6, const float* quat,
                     const float* scale, const float* view, const float* K,
                     int W, int H, float eps2d, float near_plane,
                     float far_plane, int camera_model, float mean2d[2],
                     float* depth, float conic[3], float cov2d_out[4],
                     float* comp) {
  float R[9], t[3];
  view_rt(view, R, t);
  const float mc[3] = {
      R[0] * mean_w[0] + R[1] * mean_w[1] + R[2] * mean_w[2] + t[0],
      R[3] * mean_w[0] + R[4] * mean_w[1] + R[5] * mean_w[2] + t[1],
      R[6] * mean_w[0] + R[7] * mean_w[1] + R[8] * mean_w[2] + t[2]};
  if (mc[2] < near_plane || mc[2] > far_plane) return 0;
  float cw[9], tmp[9], Rt[9], cc[9];
  if (covar6) read_covar6(covar6, cw);
  else proj_covar_from_qs(quat, scale, cw);
  m3_mul(R, cw, tmp);
  m3_t(R, Rt);
  m3_mul(tmp, Rt, cc);
  const float fx = K[0], fy = K[4], cx = K[2], cy = K[5];
  const float x = mc[0], y = mc[1], z = mc[2];
  float J[6];
  if (camera_model == 1) {
    J[0] = fx; J[1] = 0.0f; J[2] = 0.0f;
    J[3] = 0.0f; J[4] = fy; J[5] = 0.0f;
    mean2d[0] = fx * x + cx;
    mean2d[1] = fy * y + cy;
  } else if (camera_model == 2) {
    const float eps = 0.0000001f;
    const float xy_len = sqrtf(x * x + y * y) + eps;
    const float theta = atan2f(xy_len, z + eps);
    mean2d[0] = x * fx * theta / xy_len + cx;
    mean2d[1] = y * fy * theta / xy_len + cy;
    const float x2 = x * x + eps, y2 = y * y, xy = x * y;
    const float x2y2 = x2 + y2;
    const float x2y2z2_inv = 1.0f / (x2y2 + z * z);
    const float b = atan2f(xy_len, z) / xy_len / x2y2;
    const float a = z * x2y2z2_inv / x2y2;
    J[0] = fx * (x2 * a + y2 * b); J[1] = fx * xy * (a - b); J[2] = -fx * x * x2y2z2_inv;
    J[3] = fy * xy * (a - b); J[4] = fy * (y2 * a + x2 * b); J[5] = -fy * y * x2y2z2_inv;
  } else {
    const float rz = 1.0f / z, rz2 = rz * rz;
    const float tan_fovx = 0.5f * (float)W / fx;
    const float tan_fovy = 0.5f * (float)H / fy;
    const float lim_x_pos = ((float)W - cx) / fx + 0.3f * tan_fovx;
    const float lim_x_neg = cx / fx + 0.3f * tan_fovx;
    const float lim_y_pos = ((float)H - cy) / fy + 0.3f * tan_fovy;
    const float lim_y_neg = cy / fy + 0.3f * tan_fovy;
    const float tx = z * fminf(lim_x_pos, fmaxf(-lim_x_neg, x * rz));
    const float ty = z * fminf(lim_y_pos, fmaxf(-lim_y_neg, y * rz));
    J[0] = fx * rz; J[1] = 0.0f; J[2] = -fx * tx * rz2;
    J[3] = 0.0f; J[4] = fy * rz; J[5] = -fy * ty * rz2;
    mean2d[0] = fx * x * rz + cx;
    mean2d[1] = fy * y * rz + cy;
  }
  float cov2d[4] = {0, 0, 0, 0};
  for (int r = 0; r < 2; ++r)
    for (int c = 0; c < 2; ++c)
      for (int a = 0; a < 3; ++a)
        for (int b = 0; b < 3; ++b)
          cov2d[r * 2 + c] += J[r * 3 + a] * cc[a * 3 + b] * J[c * 3 + b];
  const float det_orig = cov2d[0] * cov2d[3] - cov2d[1] * cov2d[2];
  cov2d[0] += eps2d;
  cov2d[3] += eps2d;
  const float det = cov2d[0] * cov2d[3] - cov2d[1] * cov2d[2];
  if (det <= 0.0f) return 0;
  const float inv_det = 1.0f / det;
  *depth = z;
  conic[0] = cov2d[3] * inv_det;
  conic[1] = -cov2d[1] * inv_det;
  conic[2] = cov2d[0] * inv_det;
  for (int i = 0; i < 4; ++i) cov2d_out[i] = cov2d[i];
  *comp = sqrtf(fmaxf(0.005f * 0.005f, det_orig / det));
  return 1;
}

/* gsplat_projection.cpp:872-963 with metal/gsplat_projection.metal:298-338 culling. */
int orc_proj_fwd(int B, int C, int N, const float* means, const float* covars,
                 const float* quats, const float* scales,
                 const float* opacities, const float* viewmats, const float* Ks,
                 int width, int height, float eps2d, float near_plane,
                 float far_plane, float radius_clip, int calc_compensations,
                 int camera_model, float* means2d, float* depths,
                 float* conics, float* compensations, int32_t* radii) {
  if (B < 0 || C < 0 || N < 0) return ORC_ERR_ARG;
  if (!covars && (!quats || !scales)) return ORC_ERR_ARG;
  const int64_t total = (int64_t)B * C * N;
  memset(means2d, 0, sizeof(float) * 2 * total);
  memset(depths, 0, sizeof(float) * total);
  memset(conics, 0, sizeof(float) * 3 * total);
  memset(radii, 0, sizeof(int32_t) * 2 * total);
  if (calc_compensations && compensations) memset(compensations, 0, sizeof(float) * total);
  const float kAlpha = 1.0f / 255.0f;
  for (int b = 0; b < B; ++b)
    for (int c = 0; c < C; ++c)
      for (int n = 0; n < N; ++n) {
        const int64_t idx = ((int64_t)b * C + c) * N + n;
        const int64_t g = (int64_t)b * N + n;
        float m2[2], depth, conic[3], cov2d[4], comp;
        if (!proj_eval(means + g * 3, covars ? covars + g * 6 : NULL,
                       quats ? quats + g * 4 : NULL, scales ? scales + g * 3 : NULL,
                       viewmats + ((int64_t)b * C + c) * 16,
                       Ks + ((int64_t)b * C + c) * 9, width, height, eps2d,
                       near_plane, far_plane, camera_model, m2, &depth, conic,
                       cov2d, &comp))
          continue;
        float extend = 3.33f;
        if (opacities) {
          float op = opacities[g];
          if (calc_compensations) op *= comp;
          if (op < kAlpha) continue;
          extend = fminf(3.33f, sqrtf(2.0f * logf(op / kAlpha)));
        }
        const float rx = ceilf(extend * sqrtf(cov2d[0]));
        const float ry = ceilf(extend * sqrtf(cov2d[3]));
        /* metal:314 uses && (the CPU path, cpp:946, uses ||). */
        if (rx <= radius_clip && ry <= radius_clip) continue;
        /* metal:319-326: footprint entirely off the image. */
        if (m2[0] + rx <= 0.0f || m2[0] - rx >= (float)width ||
            m2[1] + ry <= 0.0f || m2[1] - ry >= (float)height)
          continue;
        radii[idx * 2] = (int32_t)rx;
        radii[idx * 2 + 1] = (int32_t)ry;
        means2d[idx * 2] = m2[0];
        means2d[idx * 2 + 1] = m2[1];
        depths[idx] = depth;
        conics[idx * 3] = conic[0];
        conics[idx * 3 + 1] = conic[1];
        conics[idx * 3 + 2] = conic[2];
        if (calc_compensations && compensations) compensations[idx] = comp;
      }
  return 0;
}

/* gsplat_projection.cpp:277-296 */
static void add_blur_vjp(float eps2d, const float cb[4], float comp,
                         float v_comp, float vc[4]) {
  const float det = cb[0] * cb[3] - cb[1] * cb[2];
  const float v_sqr = v_comp * 0.5f / (comp + 1.0e-6f);
  const float om = 1.0f - comp * comp;
  vc[0] += v_sqr * (om * cb[0] - eps2d * det);
  vc[1] += v_sqr * (om * cb[1]);
  vc[2] += v_sqr * (om * cb[2]);
  vc[3] += v_sqr * (om * cb[3] - eps2d * det);
}

/* gsplat_projection.cpp:298-376 */
static void persp_vjp(const float mc[3], const float cc[9], float fx, float fy,
                      float cx, float cy, int W, int H, const float vc2[4],
                      const float vm2[2], float vmc[3], float vcc[9]) {
  const float x = mc[0], y = mc[1], z = mc[2];
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
  for (int a = 0; a < 3; ++a)
    for (int b = 0; b < 3; ++b)
      for (int r = 0; r < 2; ++r)
        for (int c = 0; c < 2; ++c)
          vcc[a * 3 + b] += J[r * 3 + a] * vc2[r * 2 + c] * J[c * 3 + b];
  vmc[0] += fx * rz * vm2[0];
  vmc[1] += fy * rz * vm2[1];
  vmc[2] += -(fx * x * vm2[0] + fy * y * vm2[1]) * rz2;
  float vJ[6];
  for (int r = 0; r < 2; ++r)
    for (int a = 0; a < 3; ++a) {
      float left = 0.0f, right = 0.0f;
      for (int c = 0; c < 2; ++c)
        for (int b = 0; b < 3; ++b) {
          left += vc2[r * 2 + c] * J[c * 3 + b] * cc[a * 3 + b];
          right += vc2[c * 2 + r] * J[c * 3 + b] * cc[b * 3 + a];
        }
      vJ[r * 3 + a] = left + right;
    }
  if (x_rz <= lim_x_pos && x_rz >= -lim_x_neg) vmc[0] += -fx * rz2 * vJ[2];
  else vmc[2] += -fx * rz3 * tx * vJ[2];
  if (y_rz <= lim_y_pos && y_rz >= -lim_y_neg) vmc[1] += -fy * rz2 * vJ[5];
  else vmc[2] += -fy * rz3 * ty * vJ[5];
  vmc[2] += -fx * rz2 * vJ[0] - fy * rz2 * vJ[4] + 2.0f * fx * tx * rz3 * vJ[2] +
            2.0f * fy * ty * rz3 * vJ[5];
}

/* gsplat_projection.cpp:410-440 */
static void proj_rotmat_vjp(const float* q, const float g[9], float* vq) {
  float w = q[0], x = q[1], y = q[2], z = q[3];
  const float inv = 1.0f / sqrtf(w * w + x * x + y * y + z * z);
  w *= inv; x *= inv; y *= inv; z *= inv;
  const float vn[4] = {
      2.0f * (x * (g[7] - g[5]) + y * (g[2] - g[6]) + z * (g[3] - g[1])),
      2.0f * (-2.0f * x * (g[4] + g[8]) + y * (g[1] + g[3]) + z * (g[2] + g[6]) + w * (g[7] - g[5])),
      2.0f * (x * (g[1] + g[3]) - 2.0f * y * (g[0] + g[8]) + z * (g[5] + g[7]) + w * (g[2] - g[6])),
      2.0f * (x * (g[2] + g[6]) + y * (g[5] + g[7]) - 2.0f * z * (g[0] + g[4]) + w * (g[3] - g[1]))};
  const float qn[4] = {w, x, y, z};
  float dot = 0.0f;
  for (int i = 0; i < 4; ++i) dot += vn[i] * qn[i];
  for (int i = 0; i < 4; ++i) vq[i] += (vn[i] - dot * qn[i]) * inv;
}

/* gsplat_projection.cpp:442-474 */
static void proj_qs_vjp(const float* q, const float* s, const float vcw[9],
                        float* vq, float* vs) {
  float w = q[0], x = q[1], y = q[2], z = q[3];
  const float inv = 1.0f / sqrtf(w * w + x * x + y * y + z * z);
  w *= inv; x *= inv; y *= inv; z *= inv;
  const float x2 = x * x, y2 = y * y, z2 = z * z;
  const float xy = x * y, xz = x * z, yz = y * z;
  const float wx = w * x, wy = w * y, wz = w * z;
  const float R[9] = {1.0f - 2.0f * (y2 + z2), 2.0f * (xy - wz), 2.0f * (xz + wy),
                      2.0f * (xy + wz), 1.0f - 2.0f * (x2 + z2), 2.0f * (yz - wx),
                      2.0f * (xz - wy), 2.0f * (yz + wx), 1.0f - 2.0f * (x2 + y2)};
  float M[9];
  for (int r = 0; r < 3; ++r)
    for (int c = 0; c < 3; ++c) M[r * 3 + c] = R[r * 3 + c] * s[c];
  const float sym[9] = {vcw[0] + vcw[0], vcw[1] + vcw[3], vcw[2] + vcw[6],
                        vcw[3] + vcw[1], vcw[4] + vcw[4], vcw[5] + vcw[7],
                        vcw[6] + vcw[2], vcw[7] + vcw[5], vcw[8] + vcw[8]};
  float vM[9], vR[9];
  m3_mul(sym, M, vM);
  for (int r = 0; r < 3; ++r)
    for (int c = 0; c < 3; ++c) {
      vR[r * 3 + c] = vM[r * 3 + c] * s[c];
      vs[c] += vM[r * 3 + c] * R[r * 3 + c];
    }
  proj_rotmat_vjp(q, vR, vq);
}

/* gsplat_projection.cpp:965-1121 (plus metal:571-676 for v_viewmats, same math). */
int orc_proj_bwd(int B, int C, int N, const float* means, const float* covars,
                 const float* quats, const float* scales,
                 const float* viewmats, const float* Ks, int width, int height,
                 float eps2d, const int32_t* radii, const float* conics,
                 const float* compensations, const float* v_means2d,
                 const float* v_depths, const float* v_conics,
                 const float* v_compensations, float* v_means,
                 float* v_covars, float* v_quats, float* v_scales,
                 float* v_viewmats) {
  if (B < 0 || C < 0 || N < 0) return ORC_ERR_ARG;
  if (!covars && (!quats || !scales)) return ORC_ERR_ARG;
  memset(v_means, 0, sizeof(float) * 3 * (size_t)B * N);
  if (covars) memset(v_covars, 0, sizeof(float) * 6 * (size_t)B * N);
  else {
    memset(v_quats, 0, sizeof(float) * 4 * (size_t)B * N);
    memset(v_scales, 0, sizeof(float) * 3 * (size_t)B * N);
  }
  if (v_viewmats) memset(v_viewmats, 0, sizeof(float) * 16 * (size_t)B * C);
  for (int b = 0; b < B; ++b)
    for (int c = 0; c < C; ++c)
      for (int n = 0; n < N; ++n) {
        const int64_t idx = ((int64_t)b * C + c) * N + n;
        if (radii[idx * 2] <= 0 || radii[idx * 2 + 1] <= 0) continue;
        const int64_t g = (int64_t)b * N + n;
        const float* view = viewmats + ((int64_t)b * C + c) * 16;
        const float* K = Ks + ((int64_t)b * C + c) * 9;
        const float ci[4] = {conics[idx * 3], conics[idx * 3 + 1],
                             conics[idx * 3 + 1], conics[idx * 3 + 2]};
        const float vci[4] = {v_conics[idx * 3], 0.5f * v_conics[idx * 3 + 1],
                              0.5f * v_conics[idx * 3 + 1], v_conics[idx * 3 + 2]};
        /* v_cov2d = -(Ci Vci) Ci, gsplat_projection.cpp:1045-1048 */
        const float t0[4] = {ci[0] * vci[0] + ci[1] * vci[2], ci[0] * vci[1] + ci[1] * vci[3],
                             ci[2] * vci[0] + ci[3] * vci[2], ci[2] * vci[1] + ci[3] * vci[3]};
        float vc2[4] = {t0[0] * ci[0] + t0[1] * ci[2], t0[0] * ci[1] + t0[1] * ci[3],
                        t0[2] * ci[0] + t0[3] * ci[2], t0[2] * ci[1] + t0[3] * ci[3]};
        for (int i = 0; i < 4; ++i) vc2[i] *= -1.0f;
        if (v_compensations)
          add_blur_vjp(eps2d, ci, compensations[idx], v_compensations[idx], vc2);
        float R[9], t[3];
        view_rt(view, R, t);
        const float* mw = means + g * 3;
        float mc[3] = {R[0] * mw[0] + R[1] * mw[1] + R[2] * mw[2],
                       R[3] * mw[0] + R[4] * mw[1] + R[5] * mw[2],
                       R[6] * mw[0] + R[7] * mw[1] + R[8] * mw[2]};
        for (int i = 0; i < 3; ++i) mc[i] += t[i];
        float cw[9], tmp[9], Rt[9], cc[9];
        if (covars) read_covar6(covars + g * 6, cw);
        else proj_covar_from_qs(quats + g * 4, scales + g * 3, cw);
        m3_mul(R, cw, tmp);
        m3_t(R, Rt);
        m3_mul(tmp, Rt, cc);
        float vmc[3] = {0.0f, 0.0f, v_depths[idx]};
        float vcc[9] = {0};
        persp_vjp(mc, cc, K[0], K[4], K[2], K[5], width, height, vc2,
                  v_means2d + idx * 2, vmc, vcc);
        /* pos_w2c_vjp / covar_w2c_vjp, cpp:378-408 */
        float vR[9] = {0}, vt[3] = {0}, vmw[3];
        for (int r = 0; r < 3; ++r) {
          vt[r] += vmc[r];
          for (int cc2 = 0; cc2 < 3; ++cc2) vR[r * 3 + cc2] += vmc[r] * mw[cc2];
        }
        vmw[0] = R[0] * vmc[0] + R[3] * vmc[1] + R[6] * vmc[2];
        vmw[1] = R[1] * vmc[0] + R[4] * vmc[1] + R[7] * vmc[2];
        vmw[2] = R[2] * vmc[0] + R[5] * vmc[1] + R[8] * vmc[2];
        float a1[9], term1[9], vcct[9], term2[9], cwt[9], a3[9], vcw[9];
        m3_t(cw, cwt);
        m3_mul(vcc, R, a1);
        m3_mul(a1, cwt, term1);
        m3_t(vcc, vcct);
        m3_mul(vcct, R, a1);
        m3_mul(a1, cw, term2);
        m3_mul(Rt, vcc, a3);
        m3_mul(a3, R, vcw);
        for (int i = 0; i < 9; ++i) vR[i] += term1[i] + term2[i];
        for (int a = 0; a < 3; ++a) v_means[g * 3 + a] += vmw[a];
        if (covars) {
          float* o = v_covars + g * 6;
          o[0] += vcw[0];
          o[1] += vcw[1] + vcw[3];
          o[2] += vcw[2] + vcw[6];
          o[3] += vcw[4];
          o[4] += vcw[5] + vcw[7];
          o[5] += vcw[8];
        } else {
          proj_qs_vjp(quats + g * 4, scales + g * 3, vcw, v_quats + g * 4,
                      v_scales + g * 3);
        }
        if (v_viewmats) {
          float* vv = v_viewmats + ((int64_t)b * C + c) * 16;
          for (int r = 0; r < 3; ++r) {
            for (int cc2 = 0; cc2 < 3; ++cc2) vv[r * 4 + cc2] += vR[r * 3 + cc2];
            vv[r * 4 + 3] += vt[r];
          }
        }
      }
  return 0;
}

/* ------------------------------------------------------------------ */
/* spherical harmonics                                                 */
/* ------------------------------------------------------------------ */

#define SH_C0 0.2820947917738781f
#define SH_C1 0.48860251190292f

/* gsplat_spherical_harmonics.cpp:116-187 */
static void sh_basis(int degree, const float* d, float basis[25]) {
  const int cnt = (degree + 1) * (degree + 1);
  for (int i = 0; i < cnt; ++i) basis[i] = 0.0f;
  basis[0] = SH_C0;
  if (degree < 1) return;
  const float norm = sqrtf(d[0] * d[0] + d[1] * d[1] + d[2] * d[2]);
  if (norm == 0.0f) return;
  const float x = d[0] / norm, y = d[1] / norm, z = d[2] / norm;
  basis[1] = -SH_C1 * y;
  basis[2] = SH_C1 * z;
  basis[3] = -SH_C1 * x;
  if (degree < 2) return;
  const float z2 = z * z;
  const float t0b = -1.092548430592079f * z;
  const float c1 = x * x - y * y, s1 = 2.0f * x * y;
  basis[4] = 0.5462742152960395f * s1;
  basis[5] = t0b * y;
  basis[6] = 0.9461746957575601f * z2 - 0.3153915652525201f;
  basis[7] = t0b * x;
  basis[8] = 0.5462742152960395f * c1;
  if (degree < 3) return;
  const float t0c = -2.285228997322329f * z2 + 0.4570457994644658f;
  const float t1b = 1.445305721320277f * z;
  const float c2 = x * c1 - y * s1, s2 = x * s1 + y * c1;
  basis[9] = -0.5900435899266435f * s2;
  basis[10] = t1b * s1;
  basis[11] = t0c * y;
  basis[12] = z * (1.865881662950577f * z2 - 1.119528997770346f);
  basis[13] = t0c * x;
  basis[14] = t1b * c1;
  basis[15] = -0.5900435899266435f * c2;
  if (degree < 4) return;
  const float t0d = z * (-4.683325804901025f * z2 + 2.007139630671868f);
  const float t1c = 3.31161143515146f * z2 - 0.47308734787878f;
  const float t2b = -1.770130769779931f * z;
  const float c3 = x * c2 - y * s2, s3 = x * s2 + y * c2;
  basis[16] = 0.6258357354491763f * s3;
  basis[17] = t2b * s2;
  basis[18] = t1c * s1;
  basis[19] = t0d * y;
  basis[20] = 1.984313483298443f * z * basis[12] - 1.006230589874905f * basis[6];
  basis[21] = t0d * x;
  basis[22] = t1c * c1;
  basis[23] = t2b * c2;
  basis[24] = 0.6258357354491763f * c3;
}

/* gsplat_spherical_harmonics.cpp:189-286: colour = sum_b basis_b * coeff_b. */
static float sh_color(int degree, int ch, const float* d, const float* co) {
  float result = SH_C0 * co[ch];
  if (degree < 1) return result;
  const float norm = sqrtf(d[0] * d[0] + d[1] * d[1] + d[2] * d[2]);
  if (norm == 0.0f) return result;
  const float x = d[0] / norm, y = d[1] / norm, z = d[2] / norm;
  result += SH_C1 * (-y * co[3 + ch] + z * co[6 + ch] - x * co[9 + ch]);
  if (degree < 2) return result;
  const float z2 = z * z;
  const float t0b = -1.092548430592079f * z;
  const float c1 = x * x - y * y, s1 = 2.0f * x * y;
  const float p6 = 0.9461746957575601f * z2 - 0.3153915652525201f;
  const float p7 = t0b * x, p5 = t0b * y;
  const float p8 = 0.5462742152960395f * c1, p4 = 0.5462742152960395f * s1;
  result += p4 * co[12 + ch] + p5 * co[15 + ch] + p6 * co[18 + ch] +
            p7 * co[21 + ch] + p8 * co[24 + ch];
  if (degree < 3) return result;
  const float t0c = -2.285228997322329f * z2 + 0.4570457994644658f;
  const float t1b = 1.445305721320277f * z;
  const float c2 = x * c1 - y * s1, s2 = x * s1 + y * c1;
  const float p12 = z * (1.865881662950577f * z2 - 1.119528997770346f);
  const float p13 = t0c * x, p11 = t0c * y;
  const float p14 = t1b * c1, p10 = t1b * s1;
  const float p15 = -0.5900435899266435f * c2, p9 = -0.5900435899266435f * s2;
  result += p9 * co[27 + ch] + p10 * co[30 + ch] + p11 * co[33 + ch] +
            p12 * co[36 + ch] + p13 * co[39 + ch] + p14 * co[42 + ch] +
            p15 * co[45 + ch];
  if (degree < 4) return result;
  const float t0d = z * (-4.683325804901025f * z2 + 2.007139630671868f);
  const float t1c = 3.31161143515146f * z2 - 0.47308734787878f;
  const float t2b = -1.770130769779931f * z;
  const float c3 = x * c2 - y * s2, s3 = x * s2 + y * c2;
  const float p20 = 1.984313483298443f * z * p12 - 1.006230589874905f * p6;
  const float p21 = t0d * x, p19 = t0d * y;
  const float p22 = t1c * c1, p18 = t1c * s1;
  const float p23 = t2b * c2, p17 = t2b * s2;
  const float p24 = 0.6258357354491763f * c3, p16 = 0.6258357354491763f * s3;
  result += p16 * co[48 + ch] + p17 * co[51 + ch] + p18 * co[54 + ch] +
            p19 * co[57 + ch] + p20 * co[60 + ch] + p21 * co[63 + ch] +
            p22 * co[66 + ch] + p23 * co[69 + ch] + p24 * co[72 + ch];
  return result;
}

/* gsplat_spherical_harmonics.cpp:288-425: analytic d colour / d dir. */
static void sh_dir_vjp(int degree, const float* d, const float* co,
                       const float* vc, float vd[3]) {
  vd[0] = vd[1] = vd[2] = 0.0f;
  if (degree < 1) return;
  const float norm = sqrtf(d[0] * d[0] + d[1] * d[1] + d[2] * d[2]);
  if (norm == 0.0f) return;
  const float inorm = 1.0f / norm;
  const float x = d[0] * inorm, y = d[1] * inorm, z = d[2] * inorm;
  float dx[25] = {0}, dy[25] = {0}, dz[25] = {0};
  dx[3] = -SH_C1;
  dy[1] = -SH_C1;
  dz[2] = SH_C1;
  const float z2 = z * z;
  const float t0b = -1.092548430592079f * z;
  const float c1 = x * x - y * y, s1 = 2.0f * x * y;
  const float t0b_z = -1.092548430592079f;
  const float c1_x = 2.0f * x, c1_y = -2.0f * y;
  const float s1_x = 2.0f * y, s1_y = 2.0f * x;
  const float p6_z = 2.0f * 0.9461746957575601f * z;
  if (degree >= 2) {
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
  if (degree >= 3) {
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
  if (degree >= 4) {
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
  const int active = (degree + 1) * (degree + 1);
  float vn[3] = {0.0f, 0.0f, 0.0f};
  for (int b = 1; b < active; ++b) {
    const float vb = co[b * 3] * vc[0] + co[b * 3 + 1] * vc[1] + co[b * 3 + 2] * vc[2];
    vn[0] += dx[b] * vb;
    vn[1] += dy[b] * vb;
    vn[2] += dz[b] * vb;
  }
  const float dot = vn[0] * x + vn[1] * y + vn[2] * z;
  vd[0] = (vn[0] - dot * x) * inorm;
  vd[1] = (vn[1] - dot * y) * inorm;
  vd[2] = (vn[2] - dot * z) * inorm;
}

/* gsplat_spherical_harmonics.cpp:42-73 (degree and K checks) and :466-501 */
int orc_sh_fwd(int64_t n, int K, int degree, const float* dirs,
               const float* coeffs, const uint8_t* masks, float* colors) {
  if (n < 0 || degree < 0 || degree > 4 || K < (degree + 1) * (degree + 1))
    return ORC_ERR_ARG;
  for (int64_t e = 0; e < n; ++e) {
    if (masks && !masks[e]) {
      colors[e * 3] = colors[e * 3 + 1] = colors[e * 3 + 2] = 0.0f;
      continue;
    }
    for (int ch = 0; ch < 3; ++ch)
      colors[e * 3 + ch] = sh_color(degree, ch, dirs + e * 3, coeffs + e * (int64_t)K * 3);
  }
  return 0;
}

/* gsplat_spherical_harmonics.cpp:503-554 */
int orc_sh_bwd(int64_t n, int K, int degree, const float* dirs,
               const float* coeffs, const uint8_t* masks,
               const float* v_colors, float* v_dirs, float* v_coeffs) {
  if (n < 0 || degree < 0 || degree > 4 || K < (degree + 1) * (degree + 1))
    return ORC_ERR_ARG;
  memset(v_coeffs, 0, sizeof(float) * (size_t)n * K * 3);
  if (v_dirs) memset(v_dirs, 0, sizeof(float) * (size_t)n * 3);
  const int active = (degree + 1) * (degree + 1);
  float basis[25];
  for (int64_t e = 0; e < n; ++e) {
    if (masks && !masks[e]) continue;
    const float* vc = v_colors + e * 3;
    float* vco = v_coeffs + e * (int64_t)K * 3;
    sh_basis(degree, dirs + e * 3, basis);
    for (int b = 0; b < active; ++b)
      for (int ch = 0; ch < 3; ++ch) vco[b * 3 + ch] = basis[b] * vc[ch];
    if (v_dirs) sh_dir_vjp(degree, dirs + e * 3, coeffs + e * (int64_t)K * 3, vc, v_dirs + e * 3);
  }
  return 0;
}

/* ------------------------------------------------------------------ */
/* tile intersection                                                   */
/* ------------------------------------------------------------------ */

/* gsplat_intersect.cpp:60-65 */
static int floor_log2_plus_one(int v) {
  return (int)floorf(log2f((float)v)) + 1;
}

static int imin(int a, int b) { return a < b ? a : b; }
static int imax(int a, int b) { return a > b ? a : b; }

/* gsplat_intersect.cpp:67-99 */
static void tile_rect(float mx, float my, int rx, int ry, int ts, int tw, int th,
                      int rect[4]) {
  if (rx <= 0 || ry <= 0) {
    rect[0] = rect[1] = rect[2] = rect[3] = 0;
    return;
  }
  const float trx = (float)rx / (float)ts, try_ = (float)ry / (float)ts;
  const float tx = mx / (float)ts, ty = my / (float)ts;
  rect[0] = imin(imax(0, (int)floorf(tx - trx)), tw);
  rect[1] = imin(imax(0, (int)floorf(ty - try_)), th);
  rect[2] = imin(imax(0, (int)ceilf(tx + trx)), tw);
  rect[3] = imin(imax(0, (int)ceilf(ty + try_)), th);
}

/* gsplat_intersect.cpp:174-194 (checks) and :309-339 */
int orc_isect_count(int I, int N, const float* means2d, const int32_t* radii,
                    int tile_size, int tile_width, int tile_height,
                    int32_t* tiles_per_gauss) {
  if (I <= 0 || N < 0 || tile_size <= 0) return ORC_ERR_ARG;
  const int64_t n = (int64_t)I * N;
  for (int64_t i = 0; i < n; ++i) {
    int rect[4];
    tile_rect(means2d[i * 2], means2d[i * 2 + 1], radii[i * 2], radii[i * 2 + 1],
              tile_size, tile_width, tile_height, rect);
    tiles_per_gauss[i] = (rect[3] - rect[1]) * (rect[2] - rect[0]);
  }
  return 0;
}

/* gsplat_intersect.cpp:196-211 (exclusive cumsum) and :155-170 (total). */
int64_t orc_isect_scan(int64_t n, const int32_t* counts, int32_t* offsets) {
  int64_t run = 0;
  for (int64_t i = 0; i < n; ++i) {
    offsets[i] = (int32_t)run;
    run += counts[i];
  }
  return run;
}

/* gsplat_intersect.cpp:101-112 */
static int64_t encode_key(int image_id, int tile_id, float depth, int tile_bits) {
  uint32_t bits;
  memcpy(&bits, &depth, sizeof(bits));
  return ((int64_t)image_id << (32 + tile_bits)) | ((int64_t)tile_id << 32) |
         (int64_t)bits;
}

/* gsplat_intersect.cpp:213-264 (checks) and :433-485 */
int orc_isect_encode(int I, int N, const float* means2d, const int32_t* radii,
                     const float* depths, const int32_t* offsets,
                     int tile_size, int tile_width, int tile_height,
                     int64_t n_isects, int64_t* isect_ids,
                     int32_t* flatten_ids) {
  if (I <= 0 || N < 0 || tile_size <= 0 || n_isects < 0) return ORC_ERR_ARG;
  const int n_tiles = tile_width * tile_height;
  if (n_tiles <= 0) return ORC_ERR_ARG;
  const int tile_bits = floor_log2_plus_one(n_tiles);
  const int image_bits = floor_log2_plus_one(I);
  if (image_bits + tile_bits > 32) return ORC_ERR_VALUE;
  memset(isect_ids, 0, sizeof(int64_t) * (size_t)n_isects);
  memset(flatten_ids, 0, sizeof(int32_t) * (size_t)n_isects);
  const int64_t n = (int64_t)I * N;
  for (int64_t i = 0; i < n; ++i) {
    const int image_id = (int)(i / N);
    int rect[4];
    tile_rect(means2d[i * 2], means2d[i * 2 + 1], radii[i * 2], radii[i * 2 + 1],
              tile_size, tile_width, tile_height, rect);
    int64_t out = offsets[i];
    for (int ty = rect[1]; ty < rect[3]; ++ty)
      for (int tx = rect[0]; tx < rect[2]; ++tx) {
        if (out < 0 || out >= n_isects) return ORC_ERR_OOB;
        isect_ids[out] = encode_key(image_id, ty * tile_width + tx, depths[i], tile_bits);
        flatten_ids[out] = (int32_t)i;
        ++out;
      }
  }
  return 0;
}

/* Stable merge sort of (key, value) pairs by signed key. */
static void merge_pass(const int64_t* k, const int32_t* v, int64_t* k2,
                       int32_t* v2, int64_t n, int64_t w) {
  for (int64_t lo = 0; lo < n; lo += 2 * w) {
    int64_t mid = lo + w < n ? lo + w : n;
    int64_t hi = lo + 2 * w < n ? lo + 2 * w : n;
    int64_t a = lo, b = mid, o = lo;
    while (a < mid && b < hi) {
      if (k[b] < k[a]) { k2[o] = k[b]; v2[o++] = v[b++]; }
      else { k2[o] = k[a]; v2[o++] = v[a++]; }
    }
    while (a < mid) { k2[o] = k[a]; v2[o++] = v[a++]; }
    while (b < hi) { k2[o] = k[b]; v2[o++] = v[b++]; }
  }
}

/* gsplat_intersect.cpp:266-286: argsort (stable) + take of both arrays. */
int orc_isect_sort(int64_t n, const int64_t* isect_ids,
                   const int32_t* flatten_ids, int64_t* sorted_ids,
                   int32_t* sorted_flatten) {
  if (n < 0) return ORC_ERR_ARG;
  if (n == 0) return 0;
  int64_t* tk = (int64_t*)malloc(sizeof(int64_t) * (size_t)n);
  int32_t* tv = (int32_t*)malloc(sizeof(int32_t) * (size_t)n);
  if (!tk || !tv) { free(tk); free(tv); return ORC_ERR_NOMEM; }
  memcpy(sorted_ids, isect_ids, sizeof(int64_t) * (size_t)n);
  memcpy(sorted_flatten, flatten_ids, sizeof(int32_t) * (size_t)n);
  int64_t *src_k = sorted_ids, *dst_k = tk;
  int32_t *src_v = sorted_flatten, *dst_v = tv;
  for (int64_t w = 1; w < n; w *= 2) {
    merge_pass(src_k, src_v, dst_k, dst_v, n, w);
    int64_t* sk = src_k; src_k = dst_k; dst_k = sk;
    int32_t* sv = src_v; src_v = dst_v; dst_v = sv;
  }
  if (src_k != sorted_ids) {
    memcpy(sorted_ids, src_k, sizeof(int64_t) * (size_t)n);
    memcpy(sorted_flatten, src_v, sizeof(int32_t) * (size_t)n);
  }
  free(tk);
  free(tv);
  return 0;
}

/* gsplat_intersect.cpp:605-641: lower bound of (image<<tile_bits | tile). */
int orc_isect_offset(int64_t n_isects, const int64_t* isect_ids, int I,
                     int tile_width, int tile_height, int32_t* offsets) {
  if (I <= 0 || tile_width <= 0 || tile_height <= 0) return ORC_ERR_ARG;
  const int n_tiles = tile_width * tile_height;
  const int tile_bits = floor_log2_plus_one(n_tiles);
  const int64_t n_off = (int64_t)I * n_tiles;
  for (int64_t o = 0; o < n_off; ++o) {
    const int64_t key = ((o / n_tiles) << tile_bits) | (o % n_tiles);
    int64_t lo = 0, hi = n_isects;
    while (lo < hi) {
      const int64_t mid = lo + (hi - lo) / 2;
      if ((isect_ids[mid] >> 32) < key) lo = mid + 1;
      else hi = mid;
    }
    offsets[o] = (int32_t)lo;
  }
  return 0;
}

/* ------------------------------------------------------------------ */
/* rasterize                                                           */
/* ------------------------------------------------------------------ */

#define K_ALPHA_T (1.0f / 255.0f)
#define K_MAX_ALPHA 0.99f
#define K_T_EPS 1.0e-4f
#define K_MIN_1MA 1.0e-6f

/* One rasterization call: its inputs and outputs. */
typedef struct {
  int I, N, channels, width, height, tile_size, tile_width, tile_height;
  const float *means2d, *conics, *colors, *opacities, *backgrounds;
  const uint8_t* masks;
  const int32_t* tile_offsets;
  int64_t n_isects;
  const int32_t* flatten_ids;
  /* forward outputs */
  float *render_colors, *render_alphas;
  int32_t* last_ids;
  /* backward inputs */
  const float *render_alphas_in, *v_render_colors, *v_render_alphas;
  const int32_t* last_ids_in;
} RasterCall;

/* Gradient outputs of one backward worker. */
typedef struct {
  float *v_means2d_abs, *v_means2d, *v_conics, *v_colors, *v_opacities, *v_backgrounds;
} RasterGrads;

static void tile_range(const RasterCall* a, int64_t oi, int64_t* start, int64_t* end) {
  const int64_t per = (int64_t)a->tile_width * a->tile_height;
  *start = a->tile_offsets[oi];
  *end = (oi / per == a->I - 1 && oi % per == per - 1) ? a->n_isects : a->tile_offsets[oi + 1];
}

/* Forward of the pixels of tile `oi` (image-major tile index):
 * gsplat_rasterize.cpp:292-366 (CPU) == metal/gsplat_rasterize.metal:31-120. */
static void raster_fwd_tile(const RasterCall* a, int64_t oi) {
  const int per = a->tile_width * a->tile_height;
  const int im = (int)(oi / per), tid = (int)(oi % per);
  const int ty = tid / a->tile_width, tx = tid % a->tile_width;
  int64_t start, end;
  tile_range(a, oi, &start, &end);
  const int skip = a->masks && !a->masks[oi];
  const int ch_n = a->channels;
  for (int ly = 0; ly < a->tile_size; ++ly) {
    const int y = ty * a->tile_size + ly;
    if (y >= a->height) continue;
    for (int lx = 0; lx < a->tile_size; ++lx) {
      const int x = tx * a->tile_size + lx;
      if (x >= a->width) continue;
      const int64_t pix = ((int64_t)im * a->height + y) * a->width + x;
      const float px = (float)x + 0.5f, py = (float)y + 0.5f;
      float T = 1.0f;
      int32_t cur = 0;
      float* rc = a->render_colors + pix * ch_n;
      for (int ch = 0; ch < ch_n; ++ch) rc[ch] = 0.0f;
      for (int64_t idx = start; !skip && idx < end; ++idx) {
        const int g = a->flatten_ids[idx];
        const float dx = a->means2d[g * 2] - px, dy = a->means2d[g * 2 + 1] - py;
        const float c0 = a->conics[g * 3], c1 = a->conics[g * 3 + 1], c2 = a->conics[g * 3 + 2];
        const float sigma = 0.5f * (c0 * dx * dx + c2 * dy * dy) + c1 * dx * dy;
        const float alpha = fminf(K_MAX_ALPHA, a->opacities[g] * expf(-sigma));
        if (sigma < 0.0f || alpha < K_ALPHA_T) continue;
        const float next_T = T * (1.0f - alpha);
        if (next_T <= K_T_EPS) break;
        const float vis = alpha * T;
        for (int ch = 0; ch < ch_n; ++ch) rc[ch] += a->colors[(int64_t)g * ch_n + ch] * vis;
        cur = (int32_t)idx;
        T = next_T;
      }
      a->render_alphas[pix] = 1.0f - T;
      for (int ch = 0; ch < ch_n; ++ch) {
        const float bg = a->backgrounds ? a->backgrounds[im * ch_n + ch] : 0.0f;
        rc[ch] += T * bg;
      }
      a->last_ids[pix] = cur;
    }
  }
}

/* Per-worker scratch of the backward: the composited entries of a pixel. */
typedef struct {
  float* buf;
  int64_t cap;
  int64_t* ids;
  float *al, *vi;
} BwdScratch;

static int scratch_grow(BwdScratch* s) {
  const int64_t cap = s->cap ? s->cap * 2 : 1024;
  int64_t* ni = (int64_t*)realloc(s->ids, sizeof(int64_t) * (size_t)cap);
  if (ni) s->ids = ni;
  float* na = (float*)realloc(s->al, sizeof(float) * (size_t)cap);
  if (na) s->al = na;
  float* nv = (float*)realloc(s->vi, sizeof(float) * (size_t)cap);
  if (nv) s->vi = nv;
  if (!ni || !na || !nv) return ORC_ERR_NOMEM;
  s->cap = cap;
  return 0;
}

/* Backward of the pixels of tile `oi`, accumulated into `o`:
 * gsplat_rasterize.cpp:437-566 (CPU) == metal/gsplat_rasterize.metal:122-251. */
static int raster_bwd_tile(const RasterCall* a, int64_t oi, const RasterGrads* o, BwdScratch* s) {
  if (a->masks && !a->masks[oi]) return 0;
  const int per = a->tile_width * a->tile_height;
  const int im = (int)(oi / per), tid = (int)(oi % per);
  const int ty = tid / a->tile_width, tx = tid % a->tile_width;
  const int ch_n = a->channels;
  int64_t start, end;
  tile_range(a, oi, &start, &end);
  for (int ly = 0; ly < a->tile_size; ++ly) {
    const int y = ty * a->tile_size + ly;
    if (y >= a->height) continue;
    for (int lx = 0; lx < a->tile_size; ++lx) {
      const int x = tx * a->tile_size + lx;
      if (x >= a->width) continue;
      const int64_t pix = ((int64_t)im * a->height + y) * a->width + x;
      const int32_t bin_final = a->last_ids_in[pix];
      const float px = (float)x + 0.5f, py = (float)y + 0.5f;
      int64_t nv = 0;
      for (int64_t idx = start; idx < end && idx <= bin_final; ++idx) {
        const int g = a->flatten_ids[idx];
        const float dx = a->means2d[g * 2] - px, dy = a->means2d[g * 2 + 1] - py;
        const float c0 = a->conics[g * 3], c1 = a->conics[g * 3 + 1], c2 = a->conics[g * 3 + 2];
        const float sigma = 0.5f * (c0 * dx * dx + c2 * dy * dy) + c1 * dx * dy;
        const float vis = expf(-sigma);
        const float alpha = fminf(K_MAX_ALPHA, a->opacities[g] * vis);
        if (sigma < 0.0f || alpha < K_ALPHA_T) continue;
        if (nv == s->cap && scratch_grow(s)) return ORC_ERR_NOMEM;
        s->ids[nv] = idx;
        s->al[nv] = alpha;
        s->vi[nv] = vis;
        ++nv;
      }
      const float T_final = 1.0f - a->render_alphas_in[pix];
      float T = T_final;
      float* buf = s->buf;
      for (int ch = 0; ch < ch_n; ++ch) buf[ch] = 0.0f;
      const float v_a = a->v_render_alphas[pix];
      const float* v_c = a->v_render_colors + pix * ch_n;
      if (o->v_backgrounds)
        for (int ch = 0; ch < ch_n; ++ch) o->v_backgrounds[im * ch_n + ch] += T_final * v_c[ch];
      for (int64_t l = nv - 1; l >= 0; --l) {
        const int g = a->flatten_ids[s->ids[l]];
        const float alpha = s->al[l], vis = s->vi[l];
        const float ra = 1.0f / fmaxf(K_MIN_1MA, 1.0f - alpha);
        T *= ra;
        const float fac = alpha * T;
        for (int ch = 0; ch < ch_n; ++ch) o->v_colors[(int64_t)g * ch_n + ch] += fac * v_c[ch];
        float v_alpha = 0.0f;
        for (int ch = 0; ch < ch_n; ++ch)
          v_alpha += (a->colors[(int64_t)g * ch_n + ch] * T - buf[ch] * ra) * v_c[ch];
        v_alpha += T_final * ra * v_a;
        if (a->backgrounds) {
          float acc = 0.0f;
          for (int ch = 0; ch < ch_n; ++ch) acc += a->backgrounds[im * ch_n + ch] * v_c[ch];
          v_alpha += -T_final * ra * acc;
        }
        if (a->opacities[g] * vis <= K_MAX_ALPHA) {
          const float dx = a->means2d[g * 2] - px, dy = a->means2d[g * 2 + 1] - py;
          const float c0 = a->conics[g * 3], c1 = a->conics[g * 3 + 1], c2 = a->conics[g * 3 + 2];
          const float v_sigma = -a->opacities[g] * vis * v_alpha;
          const float vx = v_sigma * (c0 * dx + c1 * dy);
          const float vy = v_sigma * (c1 * dx + c2 * dy);
          o->v_conics[g * 3] += 0.5f * v_sigma * dx * dx;
          o->v_conics[g * 3 + 1] += v_sigma * dx * dy;
          o->v_conics[g * 3 + 2] += 0.5f * v_sigma * dy * dy;
          o->v_means2d[g * 2] += vx;
          o->v_means2d[g * 2 + 1] += vy;
          if (o->v_means2d_abs) {
            o->v_means2d_abs[g * 2] += fabsf(vx);
            o->v_means2d_abs[g * 2 + 1] += fabsf(vy);
          }
          o->v_opacities[g] += vis * v_alpha;
        }
        for (int ch = 0; ch < ch_n; ++ch) buf[ch] += a->colors[(int64_t)g * ch_n + ch] * fac;
      }
    }
  }
  return 0;
}

/* Workers take the tiles k, k + nthreads, k + 2 nthreads, ... of the
 * image-major tile order.  The forward writes disjoint pixels; backward
 * worker 0 accumulates into the outputs and every other worker into its own
 * zeroed copy, added to the outputs in worker order afterwards (so the
 * result depends on nthreads only through the order of the float sums). */
typedef struct {
  const RasterCall* a;
  RasterGrads g;
  int k, nthreads, bwd, rc;
} RasterWork;

static void* raster_worker(void* p) {
  RasterWork* w = (RasterWork*)p;
  const RasterCall* a = w->a;
  const int64_t n_tiles = (int64_t)a->I * a->tile_width * a->tile_height;
  BwdScratch s = {0};
  if (w->bwd) {
    s.buf = (float*)malloc(sizeof(float) * (size_t)a->channels);
    if (!s.buf || scratch_grow(&s)) w->rc = ORC_ERR_NOMEM;
  }
  for (int64_t oi = w->k; oi < n_tiles && !w->rc; oi += w->nthreads) {
    if (w->bwd) w->rc = raster_bwd_tile(a, oi, &w->g, &s);
    else raster_fwd_tile(a, oi);
  }
  free(s.buf);
  free(s.ids);
  free(s.al);
  free(s.vi);
  return NULL;
}

static size_t grad_floats(const RasterCall* a, int absgrad, int bg) {
  const size_t nG = (size_t)a->I * (size_t)a->N;
  return nG * (2 + 3 + (size_t)a->channels + 1 + (absgrad ? 2 : 0)) +
         (bg ? (size_t)a->I * a->channels : 0);
}

static RasterGrads grads_in(float* base, const RasterCall* a, int absgrad, int bg) {
  const size_t nG = (size_t)a->I * (size_t)a->N;
  RasterGrads g;
  g.v_means2d = base;
  g.v_conics = g.v_means2d + 2 * nG;
  g.v_colors = g.v_conics + 3 * nG;
  g.v_opacities = g.v_colors + (size_t)a->channels * nG;
  g.v_means2d_abs = absgrad ? g.v_opacities + nG : NULL;
  g.v_backgrounds = bg ? g.v_opacities + nG + (absgrad ? 2 * nG : 0) : NULL;
  return g;
}

static void add_into(float* dst, const float* src, size_t n) {
  if (!dst) return;
  for (size_t i = 0; i < n; ++i) dst[i] += src[i];
}

static int raster_run(const RasterCall* a, const RasterGrads* out, int bwd, int nthreads) {
  const int64_t n_tiles = (int64_t)a->I * a->tile_width * a->tile_height;
  if (nthreads < 1) nthreads = 1;
  if (nthreads > n_tiles) nthreads = n_tiles > 0 ? (int)n_tiles : 1;
  if (nthreads > 256) nthreads = 256;
  const int absgrad = bwd && out->v_means2d_abs != NULL;
  const int bg = bwd && out->v_backgrounds != NULL;
  RasterWork w[256];
  pthread_t th[256];
  float* priv[256] = {0};
  const size_t nf = bwd ? grad_floats(a, absgrad, bg) : 0;
  int rc = 0;
  for (int k = 0; k < nthreads; ++k) {
    w[k].a = a;
    w[k].k = k;
    w[k].nthreads = nthreads;
    w[k].bwd = bwd;
    w[k].rc = 0;
    if (bwd) {
      if (k == 0) {
        w[k].g = *out;
      } else {
        priv[k] = (float*)calloc(nf, sizeof(float));
        if (!priv[k]) { rc = ORC_ERR_NOMEM; nthreads = k; break; }
        w[k].g = grads_in(priv[k], a, absgrad, bg);
      }
    }
  }
  int started = 0;
  for (int k = 1; k < nthreads && !rc; ++k) {
    if (pthread_create(&th[k], NULL, raster_worker, &w[k]) != 0) break;
    started = k;
  }
  if (!rc) {
    /* tiles of workers that could not start run here, after worker 0's */
    raster_worker(&w[0]);
    for (int k = started + 1; k < nthreads; ++k) raster_worker(&w[k]);
  }
  for (int k = 1; k <= started; ++k) pthread_join(th[k], NULL);
  for (int k = 0; k < nthreads; ++k)
    if (w[k].rc) rc = w[k].rc;
  const size_t nG = (size_t)a->I * (size_t)a->N;
  for (int k = 1; k < nthreads && bwd && !rc; ++k) {
    const RasterGrads* g = &w[k].g;
    add_into(out->v_means2d, g->v_means2d, 2 * nG);
    add_into(out->v_conics, g->v_conics, 3 * nG);
    add_into(out->v_colors, g->v_colors, (size_t)a->channels * nG);
    add_into(out->v_opacities, g->v_opacities, nG);
    if (absgrad) add_into(out->v_means2d_abs, g->v_means2d_abs, 2 * nG);
    if (bg) add_into(out->v_backgrounds, g->v_backgrounds, (size_t)a->I * a->channels);
  }
  for (int k = 1; k < 256; ++k) free(priv[k]);
  return rc;
}

int orc_raster_fwd(int I, int N, int channels, const float* means2d,
                   const float* conics, const float* colors,
                   const float* opacities, const float* backgrounds,
                   const uint8_t* masks, int width, int height, int tile_size,
                   int tile_width, int tile_height, const int32_t* tile_offsets,
                   int64_t n_isects, const int32_t* flatten_ids,
                   float* render_colors, float* render_alphas,
                   int32_t* last_ids, int nthreads) {
  if (I <= 0 || channels <= 0 || tile_size <= 0) return ORC_ERR_ARG;
  const int64_t n_pix = (int64_t)I * height * width;
  memset(render_colors, 0, sizeof(float) * (size_t)n_pix * channels);
  memset(render_alphas, 0, sizeof(float) * (size_t)n_pix);
  memset(last_ids, 0, sizeof(int32_t) * (size_t)n_pix);
  RasterCall a = {I, N, channels, width, height, tile_size, tile_width, tile_height,
                  means2d, conics, colors, opacities, backgrounds, masks, tile_offsets,
                  n_isects, flatten_ids, render_colors, render_alphas, last_ids,
                  NULL, NULL, NULL, NULL};
  RasterGrads none = {0};
  return raster_run(&a, &none, 0, nthreads);
}

int orc_raster_bwd(int I, int N, int channels, const float* means2d,
                   const float* conics, const float* colors,
                   const float* opacities, const float* backgrounds,
                   const uint8_t* masks, int width, int height, int tile_size,
                   int tile_width, int tile_height, const int32_t* tile_offsets,
                   int64_t n_isects, const int32_t* flatten_ids,
                   const float* render_alphas, const int32_t* last_ids,
                   const float* v_render_colors, const float* v_render_alphas,
                   float* v_means2d_abs, float* v_means2d, float* v_conics,
                   float* v_colors, float* v_opacities, float* v_backgrounds,
                   int nthreads) {
  if (I <= 0 || channels <= 0 || tile_size <= 0) return ORC_ERR_ARG;
  const int64_t nG = (int64_t)I * N;
  if (v_means2d_abs) memset(v_means2d_abs, 0, sizeof(float) * 2 * (size_t)nG);
  memset(v_means2d, 0, sizeof(float) * 2 * (size_t)nG);
  memset(v_conics, 0, sizeof(float) * 3 * (size_t)nG);
  memset(v_colors, 0, sizeof(float) * (size_t)channels * nG);
  memset(v_opacities, 0, sizeof(float) * (size_t)nG);
  if (v_backgrounds) memset(v_backgrounds, 0, sizeof(float) * (size_t)I * channels);
  RasterCall a = {I, N, channels, width, height, tile_size, tile_width, tile_height,
                  means2d, conics, colors, opacities, backgrounds, masks, tile_offsets,
                  n_isects, flatten_ids, NULL, NULL, NULL,
                  render_alphas, v_render_colors, v_render_alphas, last_ids};
  RasterGrads out = {v_means2d_abs, v_means2d, v_conics, v_colors, v_opacities, v_backgrounds};
  return raster_run(&a, &out, 1, nthreads);
}

/* ------------------------------------------------------------------ */
/* training glue around SH (scanner_points_training_utils.py:1005-1034) */
/* ------------------------------------------------------------------ */

/* campos = -R^T t (camera_center_from_viewmat, :1005-1008). */
static void cam_center(const float* view, float cp[3]) {
  float R[9], t[3];
  view_rt(view, R, t);
  for (int i = 0; i < 3; ++i) cp[i] = -(R[i] * t[0] + R[3 + i] * t[1] + R[6 + i] * t[2]);
}

/* colors[c,n] = clip(SH(normalize(means[n] - campos_c)) + 0.5, 0, 1)
 * (sh_colors_for_camera, :1011-1034).  masks[c,n] == 0 writes 0. */
int orc_sh_glue_fwd(int C, int N, int K, int degree, const float* means,
                    const float* viewmats, const float* coeffs,
                    const uint8_t* masks, float* colors) {
  if (C < 0 || N < 0 || degree < 0 || degree > 4 || K < (degree + 1) * (degree + 1))
    return ORC_ERR_ARG;
  for (int c = 0; c < C; ++c) {
    float cp[3];
    cam_center(viewmats + (int64_t)c * 16, cp);
    for (int n = 0; n < N; ++n) {
      float* out = colors + ((int64_t)c * N + n) * 3;
      if (masks && !masks[(int64_t)c * N + n]) {
        out[0] = out[1] = out[2] = 0.0f;
        continue;
      }
      float u[3] = {means[n * 3] - cp[0], means[n * 3 + 1] - cp[1], means[n * 3 + 2] - cp[2]};
      const float m = fmaxf(sqrtf(u[0] * u[0] + u[1] * u[1] + u[2] * u[2]), 1.0e-8f);
      const float d[3] = {u[0] / m, u[1] / m, u[2] / m};
      for (int ch = 0; ch < 3; ++ch) {
        const float v = sh_color(degree, ch, d, coeffs + (int64_t)n * K * 3) + 0.5f;
        out[ch] = fminf(fmaxf(v, 0.0f), 1.0f);
      }
    }
  }
  return 0;
}

/* Reverse-mode of orc_sh_glue_fwd as MLX autograd forms it: clip passes the
 * cotangent where 0 < x < 1 (maximum/minimum vjp masks), SH backward gives
 * v_coeffs and v_dirs, and the normalisation u/max(|u|,1e-8) maps v_dirs to
 * v_means.  v_coeffs [N,K,3] and v_means [N,3] are summed over cameras. */
int orc_sh_glue_bwd(int C, int N, int K, int degree, const float* means,
                    const float* viewmats, const float* coeffs,
                    const uint8_t* masks, const float* v_colors_out,
                    float* v_means, float* v_coeffs) {
  if (C < 0 || N < 0 || degree < 0 || degree > 4 || K < (degree + 1) * (degree + 1))
    return ORC_ERR_ARG;
  memset(v_means, 0, sizeof(float) * 3 * (size_t)N);
  memset(v_coeffs, 0, sizeof(float) * 3 * (size_t)N * K);
  const int active = (degree + 1) * (degree + 1);
  float basis[25];
  for (int c = 0; c < C; ++c) {
    float cp[3];
    cam_center(viewmats + (int64_t)c * 16, cp);
    for (int n = 0; n < N; ++n) {
      if (masks && !masks[(int64_t)c * N + n]) continue;
      const float* co = coeffs + (int64_t)n * K * 3;
      float u[3] = {means[n * 3] - cp[0], means[n * 3 + 1] - cp[1], means[n * 3 + 2] - cp[2]};
      const float s = sqrtf(u[0] * u[0] + u[1] * u[1] + u[2] * u[2]);
      const float m = fmaxf(s, 1.0e-8f);
      const float d[3] = {u[0] / m, u[1] / m, u[2] / m};
      const float* vo = v_colors_out + ((int64_t)c * N + n) * 3;
      float vc[3];
      for (int ch = 0; ch < 3; ++ch) {
        const float x = sh_color(degree, ch, d, co) + 0.5f;
        vc[ch] = (x > 0.0f && x < 1.0f) ? vo[ch] : 0.0f;
      }
      sh_basis(degree, d, basis);
      float* vco = v_coeffs + (int64_t)n * K * 3;
      for (int b = 0; b < active; ++b)
        for (int ch = 0; ch < 3; ++ch) vco[b * 3 + ch] += basis[b] * vc[ch];
      float vd[3];
      sh_dir_vjp(degree, d, co, vc, vd);
      const float dot = vd[0] * u[0] + vd[1] * u[1] + vd[2] * u[2];
      for (int i = 0; i < 3; ++i) {
        float vu = vd[i] / m;
        if (s > 1.0e-8f) vu -= (u[i] / s) * dot / (m * m);
        v_means[n * 3 + i] += vu;
      }
    }
  }
  return 0;
}
