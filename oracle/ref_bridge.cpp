// extern "C" bridge over the reference's own C++ op front-ends
// (gsplat_core/gsplat_*.cpp, compiled in place against oracle/mlx_shim).
// TEST INFRASTRUCTURE ONLY: loaded by tests/golden/make_golden.py and by the
// CPU baseline of bench.py to run the reference's `eval_cpu` code on host
// buffers.  Nothing in the product links or loads this file.
//
// Built a second time with -DGSPLAT_SHIM_CUDA (oracle/_ref/
// libgsplat_ref_cuda.so) together with the product's eval_gpu adapter
// (gsplat-mlx_b200/adapter/): the same reference front-ends then dispatch
// every node to the adapter's eval_gpu bodies, which call the B200 library --
// the GPU test of that adapter.
//
// Every entry returns 0 on success and -1 when the reference threw; the
// message is then available from ref_last_error().  Shapes are the dense
// shapes the reference's tests use (leading [B] / [B,C] / [I] dims).
#include <cstdint>
#include <cstring>
#include <exception>
#include <string>
#include <vector>

#include "gsplat_core/include/gsplat_intersect.h"
#include "gsplat_core/include/gsplat_projection.h"
#include "gsplat_core/include/gsplat_quat_scale_to_covar.h"
#include "gsplat_core/include/gsplat_rasterize.h"
#include "gsplat_core/include/gsplat_spherical_harmonics.h"
#ifdef GSPLAT_SHIM_CUDA
#include "gsplat_b200_mlx.h"
#endif

namespace mx = mlx::core;
using gsplat_core::kCompensations;

namespace {

thread_local std::string g_last_error;

// The CPU build evaluates every node with eval_cpu; the device build
// (GSPLAT_SHIM_CUDA, with the CUDA eval_gpu adapter linked in) puts every
// front-end on a gpu stream, so that each node runs its eval_gpu.
#ifdef GSPLAT_SHIM_CUDA
constexpr mx::Device kDevice{mx::Device::gpu};
#else
constexpr mx::Device kDevice{mx::Device::cpu};
#endif

mx::array host(const void* p, mx::Shape shape, mx::Dtype dt) {
  return mx::array::from_host(p, std::move(shape), dt);
}

mx::array empty_f32() { return mx::zeros({0}, mx::float32); }

mx::array opt(const void* p, mx::Shape shape, mx::Dtype dt) {
  return p == nullptr ? mx::zeros({0}, dt) : host(p, std::move(shape), dt);
}

void copy_out(const mx::array& a, void* dst) {
  mx::detail::sync();
  if (dst != nullptr && a.nbytes() != 0) {
    std::memcpy(dst, a.data<void>(), a.nbytes());
  }
}

template <typename F>
int guarded(F&& f) {
  try {
    f();
    return 0;
  } catch (const std::exception& e) {
    g_last_error = e.what();
    return -1;
  }
}

}  // namespace

extern "C" {

const char* ref_last_error() { return g_last_error.c_str(); }

// gsplat_quat_scale_to_covar.cpp:337-354 (front-end) and :374-405 (eval_cpu).
int ref_qs2c_fwd(const float* quats, const float* scales, int n,
                 int compute_covar, int compute_preci, int triu,
                 float* covars, float* precis) {
  return guarded([&] {
    gsplat_core::QuatScaleToCovarPreciInput in = {
        .quats = host(quats, {n, 4}, mx::float32),
        .scales = host(scales, {n, 3}, mx::float32),
        .s = kDevice,
        .compute_covar = compute_covar != 0,
        .compute_preci = compute_preci != 0,
        .triu = triu != 0,
    };
    auto out = gsplat_core::gsplat_quat_scale_to_covar_preci_forward(in);
    copy_out(out[gsplat_core::kCovars], covars);
    copy_out(out[gsplat_core::kPrecis], precis);
  });
}

// gsplat_quat_scale_to_covar.cpp:356-372 and :407-468.
int ref_qs2c_bwd(const float* quats, const float* scales, const float* v_covars,
                 const float* v_precis, int n, int triu, float* v_quats,
                 float* v_scales) {
  return guarded([&] {
    mx::Shape cot = triu ? mx::Shape{n, 6} : mx::Shape{n, 3, 3};
    gsplat_core::QuatScaleToCovarPreciBackwardInput in = {
        .quats = host(quats, {n, 4}, mx::float32),
        .scales = host(scales, {n, 3}, mx::float32),
        .v_covars = opt(v_covars, cot, mx::float32),
        .v_precis = opt(v_precis, cot, mx::float32),
        .s = kDevice,
        .triu = triu != 0,
        .use_v_covars = v_covars != nullptr,
        .use_v_precis = v_precis != nullptr,
    };
    auto out = gsplat_core::gsplat_quat_scale_to_covar_preci_backward(in);
    copy_out(out[gsplat_core::kVQuats], v_quats);
    copy_out(out[gsplat_core::kVScales], v_scales);
  });
}

// gsplat_projection.cpp:584-618 (front-end) and :872-963 (eval_cpu).
int ref_proj_fwd(int B, int C, int N, const float* means, const float* covars,
                 const float* quats, const float* scales,
                 const float* opacities, const float* viewmats, const float* Ks,
                 int width, int height, float eps2d, float near_plane,
                 float far_plane, float radius_clip, int calc_compensations,
                 int camera_model, float* means2d, float* depths,
                 float* conics, float* compensations, int32_t* radii) {
  return guarded([&] {
    gsplat_core::ProjectionEWA3DGSFusedInput in = {
        .means = host(means, {B, N, 3}, mx::float32),
        .covars = opt(covars, {B, N, 6}, mx::float32),
        .quats = opt(quats, {B, N, 4}, mx::float32),
        .scales = opt(scales, {B, N, 3}, mx::float32),
        .opacities = opt(opacities, {B, N}, mx::float32),
        .viewmats = host(viewmats, {B, C, 4, 4}, mx::float32),
        .Ks = host(Ks, {B, C, 3, 3}, mx::float32),
        .viewspace_points = empty_f32(),
        .s = kDevice,
        .params = {
            .image_width = width,
            .image_height = height,
            .eps2d = eps2d,
            .near_plane = near_plane,
            .far_plane = far_plane,
            .radius_clip = radius_clip,
            .calc_compensations = calc_compensations != 0,
            .camera_model = camera_model,
            .use_covars = covars != nullptr,
            .use_opacities = opacities != nullptr,
        },
    };
    auto out = gsplat_core::gsplat_projection_ewa_3dgs_fused(in);
    copy_out(out[gsplat_core::kMeans2D], means2d);
    copy_out(out[gsplat_core::kDepths], depths);
    copy_out(out[gsplat_core::kConics], conics);
    copy_out(out[kCompensations], compensations);
    copy_out(out[gsplat_core::kRadii], radii);
  });
}

// gsplat_projection.cpp:620-652 and :965-1121, with the parameter overrides
// that the Python binding applies (binding/binding.cpp:157-169).
int ref_proj_bwd(int B, int C, int N, const float* means, const float* covars,
                 const float* quats, const float* scales,
                 const float* viewmats, const float* Ks, int width, int height,
                 float eps2d, const int32_t* radii, const float* conics,
                 const float* compensations, const float* v_means2d,
                 const float* v_depths, const float* v_conics,
                 const float* v_compensations, int viewmats_requires_grad,
                 float* v_means, float* v_covars, float* v_quats,
                 float* v_scales, float* v_viewmats) {
  return guarded([&] {
    gsplat_core::ProjectionEWA3DGSFusedBackwardInput in = {
        .means = host(means, {B, N, 3}, mx::float32),
        .covars = opt(covars, {B, N, 6}, mx::float32),
        .quats = opt(quats, {B, N, 4}, mx::float32),
        .scales = opt(scales, {B, N, 3}, mx::float32),
        .viewmats = host(viewmats, {B, C, 4, 4}, mx::float32),
        .Ks = host(Ks, {B, C, 3, 3}, mx::float32),
        .radii = host(radii, {B, C, N, 2}, mx::int32),
        .conics = host(conics, {B, C, N, 3}, mx::float32),
        .compensations = opt(compensations, {B, C, N}, mx::float32),
        .v_means2d = host(v_means2d, {B, C, N, 2}, mx::float32),
        .v_depths = host(v_depths, {B, C, N}, mx::float32),
        .v_conics = host(v_conics, {B, C, N, 3}, mx::float32),
        .v_compensations = opt(v_compensations, {B, C, N}, mx::float32),
        .s = kDevice,
        .params = {
            .image_width = width,
            .image_height = height,
            .eps2d = eps2d,
            .near_plane = -1.0e20f,
            .far_plane = 1.0e20f,
            .radius_clip = 0.0f,
            .calc_compensations = compensations != nullptr,
            .camera_model = 0,
            .use_covars = covars != nullptr,
            .use_opacities = false,
        },
        .viewmats_requires_grad = viewmats_requires_grad != 0,
    };
    auto out = gsplat_core::gsplat_projection_ewa_3dgs_fused_backward(in);
    copy_out(out[gsplat_core::kProjectionVMeans], v_means);
    copy_out(out[gsplat_core::kProjectionVCovars], v_covars);
    copy_out(out[gsplat_core::kProjectionVQuats], v_quats);
    copy_out(out[gsplat_core::kProjectionVScales], v_scales);
    copy_out(out[gsplat_core::kProjectionVViewmats], v_viewmats);
  });
}

// gsplat_spherical_harmonics.cpp:429-441 and :466-501.
int ref_sh_fwd(int n, int K, int degree, const float* dirs,
               const float* coeffs, const uint8_t* masks, float* colors) {
  return guarded([&] {
    gsplat_core::SphericalHarmonicsInput in = {
        .degrees_to_use = degree,
        .dirs = host(dirs, {n, 3}, mx::float32),
        .coeffs = host(coeffs, {n, K, 3}, mx::float32),
        .masks = opt(masks, {n}, mx::bool_),
        .s = kDevice,
        .use_masks = masks != nullptr,
    };
    auto out = gsplat_core::gsplat_spherical_harmonics_forward(in);
    copy_out(out, colors);
  });
}

// gsplat_spherical_harmonics.cpp:443-464 and :503-554.
int ref_sh_bwd(int n, int K, int degree, const float* dirs,
               const float* coeffs, const uint8_t* masks,
               const float* v_colors, int compute_v_dirs, float* v_dirs,
               float* v_coeffs) {
  return guarded([&] {
    gsplat_core::SphericalHarmonicsBackwardInput in = {
        .degrees_to_use = degree,
        .dirs = host(dirs, {n, 3}, mx::float32),
        .coeffs = host(coeffs, {n, K, 3}, mx::float32),
        .masks = opt(masks, {n}, mx::bool_),
        .v_colors = host(v_colors, {n, 3}, mx::float32),
        .s = kDevice,
        .use_masks = masks != nullptr,
        .compute_v_dirs = compute_v_dirs != 0,
    };
    auto out = gsplat_core::gsplat_spherical_harmonics_backward(in);
    copy_out(out[gsplat_core::kSHVDirs], v_dirs);
    copy_out(out[gsplat_core::kSHVCoeffs], v_coeffs);
  });
}

// gsplat_intersect.cpp:288-307: count -> exclusive cumsum -> host read of
// the total -> encode -> (stable argsort + take).  Returns the number of
// intersections through *n_isects.  When the caller's capacity is too small
// only the count is reported and nothing else is written.
int ref_isect_tile(int I, int N, const float* means2d, const int32_t* radii,
                   const float* depths, int tile_size, int tile_width,
                   int tile_height, int sort, int64_t capacity,
                   int32_t* tiles_per_gauss, int64_t* isect_ids,
                   int32_t* flatten_ids, int64_t* n_isects) {
  return guarded([&] {
    gsplat_core::IntersectTileInput in = {
        .means2d = host(means2d, {I, N, 2}, mx::float32),
        .radii = host(radii, {I, N, 2}, mx::int32),
        .depths = host(depths, {I, N}, mx::float32),
        .conics = empty_f32(),
        .opacities = empty_f32(),
        .image_ids = mx::zeros({0}, mx::int64),
        .gaussian_ids = mx::zeros({0}, mx::int64),
        .s = kDevice,
        .params = {
            .I = I,
            .tile_size = tile_size,
            .tile_width = tile_width,
            .tile_height = tile_height,
            .sort = sort != 0,
            .segmented = false,
            .packed = false,
            .use_conics = false,
            .use_opacities = false,
        },
    };
    auto out = gsplat_core::gsplat_intersect_tile(in);
    const int64_t m = static_cast<int64_t>(out[gsplat_core::kIsectIds].size());
    *n_isects = m;
    if (m > capacity) {
      return;
    }
    copy_out(out[gsplat_core::kTilesPerGauss], tiles_per_gauss);
    copy_out(out[gsplat_core::kIsectIds], isect_ids);
    copy_out(out[gsplat_core::kFlattenIds], flatten_ids);
  });
}

// gsplat_intersect.cpp:586-603 and :605-641.
int ref_isect_offset(int64_t n_isects, const int64_t* isect_ids, int I,
                     int tile_width, int tile_height, int32_t* offsets) {
  return guarded([&] {
    auto out = gsplat_core::gsplat_intersect_offset(
        host(isect_ids, {static_cast<int>(n_isects)}, mx::int64), I,
        tile_width, tile_height, kDevice);
    copy_out(out, offsets);
  });
}

// gsplat_rasterize.cpp:165-208 and :249-369.
int ref_raster_fwd(int I, int N, int channels, const float* means2d,
                   const float* conics, const float* colors,
                   const float* opacities, const float* backgrounds,
                   const uint8_t* masks, int width, int height, int tile_size,
                   int tile_width, int tile_height, const int32_t* tile_offsets,
                   int64_t n_isects, const int32_t* flatten_ids,
                   float* render_colors, float* render_alphas,
                   int32_t* last_ids) {
  return guarded([&] {
    gsplat_core::RasterizeToPixels3DGSInput in = {
        .means2d = host(means2d, {I, N, 2}, mx::float32),
        .conics = host(conics, {I, N, 3}, mx::float32),
        .colors = host(colors, {I, N, channels}, mx::float32),
        .opacities = host(opacities, {I, N}, mx::float32),
        .backgrounds = opt(backgrounds, {I, channels}, mx::float32),
        .masks = opt(masks, {I, tile_height, tile_width}, mx::bool_),
        .tile_offsets = host(tile_offsets, {I, tile_height, tile_width},
                             mx::int32),
        .flatten_ids = host(flatten_ids, {static_cast<int>(n_isects)},
                            mx::int32),
        .s = kDevice,
        .params = {
            .image_width = width,
            .image_height = height,
            .tile_size = tile_size,
            .use_backgrounds = backgrounds != nullptr,
            .use_masks = masks != nullptr,
            .packed = false,
        },
    };
    auto out = gsplat_core::gsplat_rasterize_to_pixels_3dgs(in);
    copy_out(out[gsplat_core::kRenderColors], render_colors);
    copy_out(out[gsplat_core::kRenderAlphas], render_alphas);
    copy_out(out[gsplat_core::kLastIds], last_ids);
  });
}

// gsplat_rasterize.cpp:210-247 and :371-569.
int ref_raster_bwd(int I, int N, int channels, const float* means2d,
                   const float* conics, const float* colors,
                   const float* opacities, const float* backgrounds,
                   const uint8_t* masks, int width, int height, int tile_size,
                   int tile_width, int tile_height, const int32_t* tile_offsets,
                   int64_t n_isects, const int32_t* flatten_ids,
                   const float* render_alphas, const int32_t* last_ids,
                   const float* v_render_colors, const float* v_render_alphas,
                   int absgrad, float* v_means2d_abs, float* v_means2d,
                   float* v_conics, float* v_colors, float* v_opacities,
                   float* v_backgrounds) {
  return guarded([&] {
    gsplat_core::RasterizeToPixels3DGSBackwardInput in = {
        .means2d = host(means2d, {I, N, 2}, mx::float32),
        .conics = host(conics, {I, N, 3}, mx::float32),
        .colors = host(colors, {I, N, channels}, mx::float32),
        .opacities = host(opacities, {I, N}, mx::float32),
        .backgrounds = opt(backgrounds, {I, channels}, mx::float32),
        .masks = opt(masks, {I, tile_height, tile_width}, mx::bool_),
        .tile_offsets = host(tile_offsets, {I, tile_height, tile_width},
                             mx::int32),
        .flatten_ids = host(flatten_ids, {static_cast<int>(n_isects)},
                            mx::int32),
        .render_alphas = host(render_alphas, {I, height, width, 1},
                              mx::float32),
        .last_ids = host(last_ids, {I, height, width}, mx::int32),
        .v_render_colors = host(v_render_colors, {I, height, width, channels},
                                mx::float32),
        .v_render_alphas = host(v_render_alphas, {I, height, width, 1},
                                mx::float32),
        .s = kDevice,
        .params = {
            .image_width = width,
            .image_height = height,
            .tile_size = tile_size,
            .use_backgrounds = backgrounds != nullptr,
            .use_masks = masks != nullptr,
            .packed = false,
        },
        .absgrad = absgrad != 0,
    };
    auto out = gsplat_core::gsplat_rasterize_to_pixels_3dgs_backward(in);
    copy_out(out[gsplat_core::kRasterVMeans2DAbs], v_means2d_abs);
    copy_out(out[gsplat_core::kRasterVMeans2D], v_means2d);
    copy_out(out[gsplat_core::kRasterVConics], v_conics);
    copy_out(out[gsplat_core::kRasterVColors], v_colors);
    copy_out(out[gsplat_core::kRasterVOpacities], v_opacities);
    copy_out(out[gsplat_core::kRasterVBackgrounds], v_backgrounds);
  });
}

#ifdef GSPLAT_SHIM_CUDA
// The adapter's one-Primitive stable sort (gsplat_b200_mlx::
// intersect_tile_sort), the replacement of argsort + take in
// gsplat_intersect.cpp:266-286.
int ref_b200_sort(int64_t n, int key_bits, const int64_t* isect_ids,
                  const int32_t* flatten_ids, int64_t* sorted_isect_ids,
                  int32_t* sorted_flatten_ids) {
  return guarded([&] {
    const int m = static_cast<int>(n);
    auto out = gsplat_b200_mlx::intersect_tile_sort(host(isect_ids, {m}, mx::int64),
                                                    host(flatten_ids, {m}, mx::int32),
                                                    key_bits, kDevice);
    copy_out(out[0], sorted_isect_ids);
    copy_out(out[1], sorted_flatten_ids);
  });
}
#endif

}  // extern "C"
