// Densification statistics of the reference trainer's default strategy
// (scripts/test/scanner_points_training_utils.py, ScannerDefaultStrategyRuntime),
// on device:
//
//   * accumulation (update_state, :412-451), every step: for each visible
//     (camera, Gaussian) observation -- both radii positive -- the norm of the
//     screen-space mean gradient scaled by (W/2, H/2) * cameras is added to
//     grad2d[n] and 1 to count[n], cameras in order (np.add.at's order), all
//     in fp32 without contraction, so the sums are the reference's bit for
//     bit; with max_radii, max_radii[n] = max(max_radii[n], r) where r is the
//     larger radius of the LAST camera that sees n over max(W, H) -- the
//     reference's fancy-index assignment keeps only the last duplicate;
//   * the refine masks: clone (_duplicate_high_grad_small, :556-569), split
//     (_split_high_grad_large, :639-657, over the Gaussians before this
//     refine's clones) and prune (_prune_gaussians, :706-718), with their
//     counts.  Scales are expf(log_scales) and opacities 1/(1+expf(-logit)):
//     a decision can differ from numpy's only where the value lies within a
//     few ulp of its threshold.
//
// One thread per Gaussian, grid-stride; HBM-bound elementwise work.  The
// file is compiled without FMA contraction (the sums must round like the
// CPU's).
#include "common.cuh"

namespace gsb {
namespace {

__global__ void __launch_bounds__(256) densify_accumulate_kernel(
    int C, int64_t N, float sx, float sy, float extent, const float* __restrict__ v_means2d,
    const int32_t* __restrict__ radii, float* __restrict__ grad2d, float* __restrict__ count,
    float* __restrict__ max_radii) {
  for (int64_t n = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; n < N;
       n += (int64_t)gridDim.x * blockDim.x) {
    float g = grad2d[n], k = count[n];
    float last = -1.0f;  // normalised radius of the last camera that sees n
    for (int c = 0; c < C; ++c) {
      const int64_t e = (int64_t)c * N + n;
      const int2 r = __ldg(reinterpret_cast<const int2*>(radii) + e);
      if (!(r.x > 0 && r.y > 0)) continue;
      const float2 v = __ldg(reinterpret_cast<const float2*>(v_means2d) + e);
      const float gx = __fmul_rn(v.x, sx), gy = __fmul_rn(v.y, sy);
      g = __fadd_rn(g, __fsqrt_rn(__fadd_rn(__fmul_rn(gx, gx), __fmul_rn(gy, gy))));
      k = __fadd_rn(k, 1.0f);
      last = __fdiv_rn((float)(r.x > r.y ? r.x : r.y), extent);
    }
    grad2d[n] = g;
    count[n] = k;
    if (max_radii && last >= 0.0f) max_radii[n] = fmaxf(max_radii[n], last);
  }
}

struct MaskArgs {
  int64_t n, n_original;
  int grow, prune, prune_scale3d, use_radii_grow, use_radii_prune;
  float grow_grad2d, grow_scale3d, grow_scale2d, prune_opa, prune_scale3d_t, prune_scale2d_t;
};

__global__ void __launch_bounds__(256) densify_masks_kernel(
    MaskArgs a, const float* __restrict__ grad2d, const float* __restrict__ count,
    const float* __restrict__ max_radii, const float* __restrict__ log_scales,
    const float* __restrict__ opacity_logits, uint8_t* __restrict__ clone,
    uint8_t* __restrict__ split, uint8_t* __restrict__ prune, unsigned long long* __restrict__ totals) {
  // totals: clone, split, prune (any reason), prune by opacity / scale3d / scale2d
  unsigned long long t[6] = {0, 0, 0, 0, 0, 0};
  for (int64_t n = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; n < a.n;
       n += (int64_t)gridDim.x * blockDim.x) {
    const float s0 = expf(__ldg(log_scales + n * 3)), s1 = expf(__ldg(log_scales + n * 3 + 1));
    const float s2 = expf(__ldg(log_scales + n * 3 + 2));
    const float max_scale = fmaxf(fmaxf(s0, s1), s2);
    if (a.grow) {
      const float k = __ldg(count + n);
      const float avg = k > 0.0f ? __fdiv_rn(__ldg(grad2d + n), fmaxf(k, 1.0f)) : 0.0f;
      const bool hot = avg > a.grow_grad2d;
      const bool c = hot && max_scale <= a.grow_scale3d;
      bool sp = hot && max_scale > a.grow_scale3d;
      if (a.use_radii_grow) sp = sp || __ldg(max_radii + n) > a.grow_scale2d;
      sp = sp && n < a.n_original;
      clone[n] = c;
      split[n] = sp;
      t[0] += c;
      t[1] += sp;
    }
    if (a.prune) {
      const float o = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-__ldg(opacity_logits + n))));
      const bool po = o < a.prune_opa;
      const bool p3 = a.prune_scale3d && max_scale > a.prune_scale3d_t;
      const bool p2 = a.use_radii_prune && __ldg(max_radii + n) > a.prune_scale2d_t;
      const bool any = po || p3 || p2;
      prune[n] = any;
      t[2] += any;
      t[3] += po;
      t[4] += p3;
      t[5] += p2;
    }
  }
#pragma unroll
  for (int i = 0; i < 6; ++i) {
    unsigned long long v = t[i];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if ((threadIdx.x & 31) == 0 && v) atomicAdd(totals + i, v);
  }
}

}  // namespace
}  // namespace gsb

using namespace gsb;

extern "C" int gs_densify_accumulate(const gs_densify_params* p, const float* v_means2d,
                                     const int32_t* radii, float* grad2d, float* count,
                                     float* max_radii, gs_stream_t stream) {
  if (!p || p->C <= 0 || p->N < 0 || p->width <= 0 || p->height <= 0 || p->n_cameras <= 0)
    return invalid("densify_accumulate: bad params");
  if (p->N == 0) return GS_OK;
  if (!v_means2d || !radii || !grad2d || !count) return invalid("densify_accumulate: missing buffer");
  // the reference scales by Python floats: (W / 2.0) * cameras in double,
  // then rounded to fp32 for the fp32 multiply
  const float sx = (float)((double)p->width / 2.0 * (double)p->n_cameras);
  const float sy = (float)((double)p->height / 2.0 * (double)p->n_cameras);
  const int extent = p->width > p->height ? p->width : p->height;
  densify_accumulate_kernel<<<grid_for(p->N, 256), 256, 0, as_stream(stream)>>>(
      p->C, p->N, sx, sy, (float)extent, v_means2d, radii, grad2d, count, max_radii);
  return launch_status("densify_accumulate");
}

extern "C" int gs_densify_masks(const gs_densify_mask_params* p, const float* grad2d,
                                const float* count, const float* max_radii,
                                const float* log_scales, const float* opacity_logits,
                                uint8_t* clone, uint8_t* split, uint8_t* prune,
                                int64_t* totals_device, gs_stream_t stream) {
  if (!p || p->n < 0 || p->n_original < 0) return invalid("densify_masks: bad params");
  if (!totals_device) return invalid("densify_masks: missing totals");
  cudaStream_t s = as_stream(stream);
  if (cudaMemsetAsync(totals_device, 0, 6 * sizeof(int64_t), s) != cudaSuccess)
    return launch_status("densify_masks");
  if (p->n == 0) return GS_OK;
  const bool grow = p->compute_grow != 0, prn = p->compute_prune != 0;
  // the reference's refine_scale2d_stop_iter schedule for the 2D-radius terms
  const bool radii_on = p->refine_scale2d_stop_iter > 0 && p->step < p->refine_scale2d_stop_iter;
  if (!log_scales || (grow && (!grad2d || !count || !clone || !split)) ||
      (prn && (!opacity_logits || !prune)) || (radii_on && !max_radii))
    return invalid("densify_masks: missing buffer");
  MaskArgs a;
  a.n = p->n;
  a.n_original = p->n_original;
  a.grow = grow;
  a.prune = prn;
  a.prune_scale3d = p->step > p->reset_every;
  a.use_radii_grow = radii_on && grow;
  a.use_radii_prune = radii_on && prn && p->step > p->reset_every;
  // thresholds: Python floats (products in double) compared with fp32 arrays
  a.grow_grad2d = (float)p->grow_grad2d;
  a.grow_scale3d = (float)(p->grow_scale3d * p->scene_scale);
  a.grow_scale2d = (float)p->grow_scale2d;
  a.prune_opa = (float)p->prune_opa;
  a.prune_scale3d_t = (float)(p->prune_scale3d * p->scene_scale);
  a.prune_scale2d_t = (float)p->prune_scale2d;
  densify_masks_kernel<<<grid_for(p->n, 256), 256, 0, s>>>(
      a, grad2d, count, max_radii, log_scales, opacity_logits, clone, split, prune,
      reinterpret_cast<unsigned long long*>(totals_device));
  return launch_status("densify_masks");
}
