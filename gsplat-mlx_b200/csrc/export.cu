// SPZ export attributes of the reference trainer
// (scripts/test/scanner_points_training_utils.py, export_trained_spz,
// :1424-1493): from the trained parameters, the arrays the reference hands
// to the spz package's GaussianCloud --
//   positions  (x, -z, y)                                   positions_to_spz :1361
//   scales     log-scales, or with y and z swapped           scales_to_spz :1380
//   rotations  the quaternion normalised, or taken through its rotation
//              matrix into the SPZ axes (A R, F R F^T or A R A^T) and back by
//              the largest-of-four extraction, normalised, stored wxyz or
//              xyzw                         quats_to_spz :1392, _storage :1415
//   alphas     the opacity logits
//   colors     DC coefficients, clip(0.5 + C0 dc), or from RGB colours
//              (clip(c) - 0.5) / C0 or clip(c)                        :1461-1486
//   sh         the first (degree + 1)^2 - 1 rest coefficients
// One thread per Gaussian, fp32 in the reference's operation order without
// FMA contraction; HBM-bound elementwise work.  The byte packing and gzip of
// the .spz file are the spz package's (not part of this library).
#include "common.cuh"

namespace gsb {
namespace {

constexpr float kShC0 = 0.28209479177387814f;

__device__ __forceinline__ void normalize4(float q[4]) {
  const float n = fmaxf(sqrtf(q[0] * q[0] + q[1] * q[1] + q[2] * q[2] + q[3] * q[3]), 1.0e-8f);
#pragma unroll
  for (int i = 0; i < 4; ++i) q[i] = q[i] / n;
}

// m = L r R^T for the signed axis permutations L, R (entries 0 / +-1):
// row i of L picks row li[i] of r with sign ls[i], likewise for columns.
__device__ __forceinline__ void permute3(const float r[9], const int li[3], const float ls[3],
                                         const int ri[3], const float rs[3], float m[9]) {
#pragma unroll
  for (int i = 0; i < 3; ++i)
#pragma unroll
    for (int j = 0; j < 3; ++j) m[i * 3 + j] = ls[i] * rs[j] * r[li[i] * 3 + ri[j]];
}

__device__ __forceinline__ void rot_to_quat(const float r[9], float q[4]) {
  const float tr = r[0] + r[4] + r[8];
  if (tr > 0.0f) {
    const float s = sqrtf(tr + 1.0f) * 2.0f;
    q[0] = 0.25f * s;
    q[1] = (r[7] - r[5]) / s;
    q[2] = (r[2] - r[6]) / s;
    q[3] = (r[3] - r[1]) / s;
  } else if (r[0] > r[4] && r[0] > r[8]) {
    const float s = sqrtf(1.0f + r[0] - r[4] - r[8]) * 2.0f;
    q[0] = (r[7] - r[5]) / s;
    q[1] = 0.25f * s;
    q[2] = (r[1] + r[3]) / s;
    q[3] = (r[2] + r[6]) / s;
  } else if (r[4] > r[8]) {
    const float s = sqrtf(1.0f + r[4] - r[0] - r[8]) * 2.0f;
    q[0] = (r[2] - r[6]) / s;
    q[1] = (r[1] + r[3]) / s;
    q[2] = 0.25f * s;
    q[3] = (r[5] + r[7]) / s;
  } else {
    const float s = sqrtf(1.0f + r[8] - r[0] - r[4]) * 2.0f;
    q[0] = (r[3] - r[1]) / s;
    q[1] = (r[2] + r[6]) / s;
    q[2] = (r[5] + r[7]) / s;
    q[3] = 0.25f * s;
  }
  normalize4(q);
}

struct SpzArgs {
  int64_t n;
  int scale_mode, rotation_mode, quat_order, color_mode, source, sh_rest, rest_stride;
  const float *means, *quats, *log_scales, *opacity_logits, *colors_in, *features_rest;
  float *positions, *scales, *rotations, *alphas, *colors, *sh;
};

__global__ void __launch_bounds__(256) spz_attributes_kernel(const SpzArgs a) {
  for (int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; g < a.n;
       g += (int64_t)gridDim.x * blockDim.x) {
    const float* m = a.means + g * 3;
    a.positions[g * 3] = m[0];
    a.positions[g * 3 + 1] = -m[2];
    a.positions[g * 3 + 2] = m[1];
    const float* ls = a.log_scales + g * 3;
    a.scales[g * 3] = ls[0];
    a.scales[g * 3 + 1] = a.scale_mode ? ls[2] : ls[1];
    a.scales[g * 3 + 2] = a.scale_mode ? ls[1] : ls[2];
    float q[4] = {a.quats[g * 4], a.quats[g * 4 + 1], a.quats[g * 4 + 2], a.quats[g * 4 + 3]};
    normalize4(q);
    if (a.rotation_mode != 0) {
      const float w = q[0], x = q[1], y = q[2], z = q[3];
      const float r[9] = {1.0f - 2.0f * (y * y + z * z), 2.0f * (x * y - z * w),
                          2.0f * (x * z + y * w),        2.0f * (x * y + z * w),
                          1.0f - 2.0f * (x * x + z * z), 2.0f * (y * z - x * w),
                          2.0f * (x * z - y * w),        2.0f * (y * z + x * w),
                          1.0f - 2.0f * (x * x + y * y)};
      // position axis A = [[1,0,0],[0,0,-1],[0,1,0]], fastgs axis F = A^T
      const int pi[3] = {0, 2, 1}, id[3] = {0, 1, 2};
      const float as[3] = {1.0f, -1.0f, 1.0f}, fs[3] = {1.0f, 1.0f, -1.0f};
      const float one[3] = {1.0f, 1.0f, 1.0f};
      float mr[9];
      if (a.rotation_mode == 1) permute3(r, pi, as, id, one, mr);       // A R
      else if (a.rotation_mode == 2) permute3(r, pi, fs, pi, fs, mr);   // F R F^T
      else permute3(r, pi, as, pi, as, mr);                             // A R A^T
      rot_to_quat(mr, q);
    }
    normalize4(q);
    float* ro = a.rotations + g * 4;
    if (a.quat_order) {
      ro[0] = q[1];
      ro[1] = q[2];
      ro[2] = q[3];
      ro[3] = q[0];
    } else {
      ro[0] = q[0];
      ro[1] = q[1];
      ro[2] = q[2];
      ro[3] = q[3];
    }
    a.alphas[g] = a.opacity_logits[g];
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      const float v = a.colors_in[g * 3 + c];
      float o;
      if (a.source) {  // RGB model colours
        const float cl = fminf(fmaxf(v, 0.0f), 1.0f);
        o = a.color_mode ? cl : (cl - 0.5f) / kShC0;
      } else {         // SH model DC coefficients
        o = a.color_mode ? fminf(fmaxf(0.5f + kShC0 * v, 0.0f), 1.0f) : v;
      }
      a.colors[g * 3 + c] = o;
    }
    for (int k = 0; k < a.sh_rest * 3; ++k)
      a.sh[g * a.sh_rest * 3 + k] = a.features_rest[g * (int64_t)a.rest_stride * 3 + k];
  }
}

}  // namespace
}  // namespace gsb

using namespace gsb;

extern "C" int gs_spz_attributes(const gs_spz_params* p, const float* means, const float* quats,
                                 const float* log_scales, const float* opacity_logits,
                                 const float* colors_or_dc, const float* features_rest,
                                 float* positions, float* scales, float* rotations, float* alphas,
                                 float* colors, float* sh, gs_stream_t stream) {
  if (!p || p->n < 0 || p->scale_mode < 0 || p->scale_mode > 1 || p->rotation_mode < 0 ||
      p->rotation_mode > 3 || p->quat_order < 0 || p->quat_order > 1 || p->color_mode < 0 ||
      p->color_mode > 1 || p->source < 0 || p->source > 1 || p->sh_rest < 0 ||
      p->sh_rest > p->rest_stride || (p->sh_rest > 0 && (p->source == 1 || p->color_mode == 1)))
    return invalid("spz_attributes: bad params");
  if (p->n == 0) return GS_OK;
  if (!means || !quats || !log_scales || !opacity_logits || !colors_or_dc || !positions ||
      !scales || !rotations || !alphas || !colors || (p->sh_rest > 0 && (!features_rest || !sh)))
    return invalid("spz_attributes: missing buffer");
  const SpzArgs a{p->n, p->scale_mode, p->rotation_mode, p->quat_order, p->color_mode,
                  p->source, p->sh_rest, p->rest_stride, means, quats, log_scales,
                  opacity_logits, colors_or_dc, features_rest, positions, scales, rotations,
                  alphas, colors, sh};
  spz_attributes_kernel<<<grid_for(p->n, 256), 256, 0, as_stream(stream)>>>(a);
  return launch_status("spz_attributes");
}
