// Fused training glue around the operators, for the reference's image-fitting
// trainer (scripts/test/train_image_fitting_3dgs_mlx.py) on device:
//
//   * parameter activations (:33-36, :104-118): quats / max(|quats|, 1e-8),
//     scales = exp(log_scales), colors = sigmoid(color_logits),
//     opacities = sigmoid(opacity_logits);
//   * the L2 image loss of the fitting benchmark: loss = mean((render -
//     target)^2), cotangent 2 (render - target) / count;
//   * MLX Adam (mlx.optimizers.Adam with its defaults: no bias correction)
//     applied to the raw parameters through the reverse mode of the
//     activations, then the quaternion renormalisation of the trainer (:566)
//     and the activations for the next step -- one pass over the Gaussians.
//
// All elementwise and HBM-bound: one thread per Gaussian (per image element
// for the loss), grid-stride loops.
#include "common.cuh"

namespace gsb {
namespace {

__device__ __forceinline__ float sigmoidf(float x) { return 1.0f / (1.0f + expf(-x)); }

__device__ __forceinline__ void activate_one(int64_t n, const float* __restrict__ quats,
                                             const float* __restrict__ log_scales,
                                             const float* __restrict__ color_logits,
                                             const float* __restrict__ opacity_logits,
                                             float* __restrict__ quats_n, float* __restrict__ scales,
                                             float* __restrict__ colors,
                                             float* __restrict__ opacities) {
  const float4 q = reinterpret_cast<const float4*>(quats)[n];
  const float norm = sqrtf(q.x * q.x + q.y * q.y + q.z * q.z + q.w * q.w);
  const float d = fmaxf(norm, 1.0e-8f);
  reinterpret_cast<float4*>(quats_n)[n] = make_float4(q.x / d, q.y / d, q.z / d, q.w / d);
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    scales[n * 3 + k] = expf(log_scales[n * 3 + k]);
    colors[n * 3 + k] = sigmoidf(color_logits[n * 3 + k]);
  }
  opacities[n] = sigmoidf(opacity_logits[n]);
}

__global__ void __launch_bounds__(256) fit_activate_kernel(
    int64_t N, const float* __restrict__ quats, const float* __restrict__ log_scales,
    const float* __restrict__ color_logits, const float* __restrict__ opacity_logits,
    float* __restrict__ quats_n, float* __restrict__ scales, float* __restrict__ colors,
    float* __restrict__ opacities) {
  for (int64_t n = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; n < N;
       n += (int64_t)gridDim.x * blockDim.x)
    activate_one(n, quats, log_scales, color_logits, opacity_logits, quats_n, scales, colors,
                 opacities);
}

// v = 2 (render - target) / count; loss += sum (render - target)^2 / count.
__global__ void __launch_bounds__(256) l2_loss_grad_kernel(int64_t count,
                                                           const float* __restrict__ render,
                                                           const float* __restrict__ target,
                                                           float* __restrict__ v_render,
                                                           float* __restrict__ loss) {
  const float inv = 1.0f / (float)count;
  float acc = 0.0f;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float d = __ldg(render + i) - __ldg(target + i);
    v_render[i] = 2.0f * d * inv;
    acc += d * d;
  }
  __shared__ float s_part[8];
  acc = warp_sum(acc);
  if ((threadIdx.x & 31) == 0) s_part[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.0f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += s_part[w];
    atomicAdd(loss, t * inv);
  }
}

struct AdamHP {
  float lr, b1, b2, eps;
};

__device__ __forceinline__ float adam(float p, float g, float& m, float& v, const AdamHP& h) {
  m = h.b1 * m + (1.0f - h.b1) * g;
  v = h.b2 * v + (1.0f - h.b2) * g * g;
  return p - h.lr * m / (sqrtf(v) + h.eps);
}

// Reverse mode of the activations, Adam on the raw parameters, quaternion
// renormalisation, activations for the next step.  Moments m/v hold, per
// Gaussian, [means 3 | quats 4 | log_scales 3 | color_logits 3 | opacity 1].
__global__ void __launch_bounds__(256) fit_adam_kernel(
    int64_t N, AdamHP h, float* __restrict__ means, float* __restrict__ quats,
    float* __restrict__ log_scales, float* __restrict__ color_logits,
    float* __restrict__ opacity_logits, const float* __restrict__ v_means,
    const float* __restrict__ v_quats_n, const float* __restrict__ v_scales,
    const float* __restrict__ v_colors, const float* __restrict__ v_opacities,
    float* __restrict__ m1, float* __restrict__ m2, float* __restrict__ quats_n,
    float* __restrict__ scales, float* __restrict__ colors, float* __restrict__ opacities) {
  for (int64_t n = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; n < N;
       n += (int64_t)gridDim.x * blockDim.x) {
    float* mm = m1 + n * 14;
    float* vv = m2 + n * 14;
#pragma unroll
    for (int k = 0; k < 3; ++k)
      means[n * 3 + k] = adam(means[n * 3 + k], v_means[n * 3 + k], mm[k], vv[k], h);
    // quats: d(q / max(|q|, eps)) -- (g - qn (qn . g)) / |q| above eps, g / eps below
    const float4 q = reinterpret_cast<const float4*>(quats)[n];
    const float qa[4] = {q.x, q.y, q.z, q.w};
    const float norm = sqrtf(q.x * q.x + q.y * q.y + q.z * q.z + q.w * q.w);
    const float d = fmaxf(norm, 1.0e-8f);
    float qn[4], g[4];
    float dot = 0.0f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      qn[k] = qa[k] / d;
      g[k] = v_quats_n[n * 4 + k];
      dot += qn[k] * g[k];
    }
    float qq[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float gr = norm > 1.0e-8f ? (g[k] - qn[k] * dot) / d : g[k] / d;
      qq[k] = adam(qa[k], gr, mm[3 + k], vv[3 + k], h);
    }
    // the trainer renormalises the raw quaternion after the update
    const float n2 = sqrtf(qq[0] * qq[0] + qq[1] * qq[1] + qq[2] * qq[2] + qq[3] * qq[3]);
    const float d2 = fmaxf(n2, 1.0e-8f);
#pragma unroll
    for (int k = 0; k < 4; ++k) qq[k] /= d2;
    reinterpret_cast<float4*>(quats)[n] = make_float4(qq[0], qq[1], qq[2], qq[3]);
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      const float s = scales[n * 3 + k];  // exp(log_scale) of this step
      log_scales[n * 3 + k] =
          adam(log_scales[n * 3 + k], v_scales[n * 3 + k] * s, mm[7 + k], vv[7 + k], h);
      const float c = colors[n * 3 + k];
      color_logits[n * 3 + k] = adam(color_logits[n * 3 + k], v_colors[n * 3 + k] * c * (1.0f - c),
                                     mm[10 + k], vv[10 + k], h);
    }
    const float o = opacities[n];
    opacity_logits[n] = adam(opacity_logits[n], v_opacities[n] * o * (1.0f - o), mm[13], vv[13], h);
    activate_one(n, quats, log_scales, color_logits, opacity_logits, quats_n, scales, colors,
                 opacities);
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace
}  // namespace gsb

using namespace gsb;

extern "C" int gs_fit_activate(int64_t n, const float* quats, const float* log_scales,
                               const float* color_logits, const float* opacity_logits,
                               float* quats_n, float* scales, float* colors, float* opacities,
                               gs_stream_t stream) {
  if (n < 0) return invalid("fit_activate: negative size");
  if (n == 0) return GS_OK;
  if (!quats || !log_scales || !color_logits || !opacity_logits || !quats_n || !scales ||
      !colors || !opacities)
    return invalid("fit_activate: missing buffer");
  if (!aligned16(quats) || !aligned16(quats_n))
    return invalid("fit_activate: quaternion buffers must be 16-byte aligned");
  fit_activate_kernel<<<grid_for(n, 256), 256, 0, as_stream(stream)>>>(
      n, quats, log_scales, color_logits, opacity_logits, quats_n, scales, colors, opacities);
  return launch_status("fit_activate");
}

extern "C" int gs_l2_loss_grad(int64_t count, const float* render, const float* target,
                               float* v_render, float* loss, gs_stream_t stream) {
  if (count < 0) return invalid("l2_loss_grad: negative size");
  if (count == 0) return GS_OK;
  if (!render || !target || !v_render || !loss) return invalid("l2_loss_grad: missing buffer");
  cudaStream_t s = as_stream(stream);
  if (cudaMemsetAsync(loss, 0, sizeof(float), s) != cudaSuccess) return launch_status("l2_loss_grad");
  l2_loss_grad_kernel<<<grid_for(count, 256), 256, 0, s>>>(count, render, target, v_render, loss);
  return launch_status("l2_loss_grad");
}

extern "C" int gs_fit_adam(const gs_adam_params* p, float* means, float* quats, float* log_scales,
                           float* color_logits, float* opacity_logits, const float* v_means,
                           const float* v_quats, const float* v_scales, const float* v_colors,
                           const float* v_opacities, float* moment1, float* moment2,
                           float* quats_n, float* scales, float* colors, float* opacities,
                           gs_stream_t stream) {
  if (!p || p->n < 0) return invalid("fit_adam: bad params");
  if (p->n == 0) return GS_OK;
  if (!means || !quats || !log_scales || !color_logits || !opacity_logits || !v_means ||
      !v_quats || !v_scales || !v_colors || !v_opacities || !moment1 || !moment2 || !quats_n ||
      !scales || !colors || !opacities)
    return invalid("fit_adam: missing buffer");
  if (!aligned16(quats) || !aligned16(quats_n))
    return invalid("fit_adam: quaternion buffers must be 16-byte aligned");
  const AdamHP h{p->learning_rate, p->beta1, p->beta2, p->eps};
  fit_adam_kernel<<<grid_for(p->n, 256), 256, 0, as_stream(stream)>>>(
      p->n, h, means, quats, log_scales, color_logits, opacity_logits, v_means, v_quats, v_scales,
      v_colors, v_opacities, moment1, moment2, quats_n, scales, colors, opacities);
  return launch_status("fit_adam");
}
