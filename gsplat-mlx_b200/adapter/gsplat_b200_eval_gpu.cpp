// The `eval_gpu` bodies of the reference's gsplat_core Primitives over the
// gsplat_b200 C ABI (see gsplat_b200_mlx.h for how a CUDA build of the
// reference takes them).  Each body replaces the Metal dispatch block named
// in its comment: it reads the same inputs in the same order, derives the
// same sizes from their shapes and the Primitive's parameters, allocates the
// outputs the front-end declared, and makes one call into the library.
//
// Compile with the reference's tree and MLX (or any MLX-compatible headers)
// on the include path, and gsplat_b200.h:
//   g++ -std=c++20 -I<reference> -I<mlx> -I<repo>/include -c gsplat_b200_eval_gpu.cpp
#include "gsplat_b200_mlx.h"

#include <algorithm>
#include <cstring>
#include <numeric>
#include <stdexcept>
#include <string>
#include <utility>

#include <cuda_runtime_api.h>

#include "gsplat_b200.h"
#include "gsplat_core/include/gsplat_intersect.h"
#include "gsplat_core/include/gsplat_projection.h"
#include "gsplat_core/include/gsplat_quat_scale_to_covar.h"
#include "gsplat_core/include/gsplat_rasterize.h"
#include "gsplat_core/include/gsplat_spherical_harmonics.h"

namespace gsplat_b200_mlx {
namespace {

StreamResolver g_resolver = nullptr;

// One launch scope: resolves the Primitive's CUDA stream; without a
// resolver waits for the device first and for the legacy stream at the end.
class Launch {
 public:
  explicit Launch(const mx::Stream& s) {
    stream_ = g_resolver != nullptr ? g_resolver(s) : nullptr;
    sync_ = stream_ == nullptr;
    if (sync_) {
      check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
    }
  }
  gs_stream_t stream() const { return stream_; }
  // Throws on a failed call; on success waits when running synchronously.
  void done(int rc, const char* op) {
    if (rc != GS_OK) {
      throw std::runtime_error(std::string(op) + ": " + gs_status_string(rc) + ": " +
                               gs_last_error());
    }
    if (sync_) {
      check_cuda(cudaStreamSynchronize(nullptr), op);
    }
  }

 private:
  static void check_cuda(cudaError_t e, const char* what) {
    if (e != cudaSuccess) {
      throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
    }
  }
  gs_stream_t stream_ = nullptr;
  bool sync_ = true;
};

void allocate(std::vector<mx::array>& outputs) {
  for (auto& out : outputs) {
    out.set_data(mx::allocator::malloc(out.nbytes()));
  }
}

template <typename T>
const T* ptr(const mx::array& a) {
  return a.size() == 0 ? nullptr : a.data<T>();
}

template <typename T>
T* out_ptr(mx::array& a) {
  return a.size() == 0 ? nullptr : a.data<T>();
}

int last_dim(const mx::array& a, int from_end) {
  return a.shape(static_cast<int>(a.ndim()) - from_end);
}

}  // namespace

void set_stream_resolver(StreamResolver resolver) { g_resolver = resolver; }

// ---------------------------------------------------------------- sort

std::vector<mx::array> intersect_tile_sort(const mx::array& isect_ids,
                                           const mx::array& flatten_ids, int key_bits,
                                           mx::StreamOrDevice s) {
  if (isect_ids.dtype().val() != mx::int64.val() ||
      flatten_ids.dtype().val() != mx::int32.val() ||
      isect_ids.ndim() != 1 || flatten_ids.ndim() != 1 ||
      isect_ids.size() != flatten_ids.size()) {
    throw std::runtime_error(
        "intersect_tile_sort expects matching 1D int64 isect_ids and int32 flatten_ids.");
  }
  if (key_bits < 1 || key_bits > 64) {
    throw std::runtime_error("intersect_tile_sort expects 1 <= key_bits <= 64.");
  }
  const int n = static_cast<int>(isect_ids.size());
  // The radix sort's scratch is a third output (int32 words) that the caller
  // drops: MLX keeps it alive until the stream has finished with it.
  const size_t ws = gs_isect_sort_workspace_size(n);
  const int ws_words = static_cast<int>((ws + 3) / 4);
  auto prim = std::make_shared<IntersectSort>(mx::to_stream(s), key_bits);
  auto outs = mx::array::make_arrays({mx::Shape{n}, mx::Shape{n}, mx::Shape{ws_words}},
                                     {mx::int64, mx::int32, mx::int32}, prim,
                                     {mx::contiguous(isect_ids), mx::contiguous(flatten_ids)});
  return {outs[0], outs[1]};
}

void IntersectSort::eval_cpu(const std::vector<mx::array>& inputs,
                             std::vector<mx::array>& outputs) {
  allocate(outputs);
  const size_t n = inputs[0].size();
  const int64_t* keys = inputs[0].data<int64_t>();
  const int32_t* ids = inputs[1].data<int32_t>();
  std::vector<size_t> order(n);
  std::iota(order.begin(), order.end(), size_t{0});
  std::stable_sort(order.begin(), order.end(),
                   [keys](size_t a, size_t b) { return keys[a] < keys[b]; });
  int64_t* ok = outputs[0].data<int64_t>();
  int32_t* oi = outputs[1].data<int32_t>();
  for (size_t i = 0; i < n; ++i) {
    ok[i] = keys[order[i]];
    oi[i] = ids[order[i]];
  }
}

void IntersectSort::eval_gpu(const std::vector<mx::array>& inputs,
                             std::vector<mx::array>& outputs) {
  allocate(outputs);
  const int64_t n = static_cast<int64_t>(inputs[0].size());
  if (n == 0) {
    return;
  }
  Launch L(stream());
  L.done(gs_isect_sort(n, key_bits_, inputs[0].data<int64_t>(), inputs[1].data<int32_t>(),
                       outputs[0].data<int64_t>(), outputs[1].data<int32_t>(),
                       outputs[2].data<int32_t>(), outputs[2].nbytes(), L.stream()),
         "intersect_tile_sort");
}

std::vector<mx::array> IntersectSort::jvp(const std::vector<mx::array>&,
                                          const std::vector<mx::array>&,
                                          const std::vector<int>&) {
  throw std::runtime_error("GSPlatB200IntersectSort has no JVP.");
}

std::vector<mx::array> IntersectSort::vjp(const std::vector<mx::array>&,
                                          const std::vector<mx::array>&,
                                          const std::vector<int>&,
                                          const std::vector<mx::array>&) {
  throw std::runtime_error("GSPlatB200IntersectSort has no VJP.");
}

std::pair<std::vector<mx::array>, std::vector<int>> IntersectSort::vmap(
    const std::vector<mx::array>&, const std::vector<int>&) {
  throw std::runtime_error("GSPlatB200IntersectSort has no vmap.");
}

bool IntersectSort::is_equivalent(const mx::Primitive& other) const {
  const auto* o = dynamic_cast<const IntersectSort*>(&other);
  return o != nullptr && o->key_bits_ == key_bits_;
}

}  // namespace gsplat_b200_mlx

namespace gsplat_core {

using gsplat_b200_mlx::Launch;
using gsplat_b200_mlx::allocate;
using gsplat_b200_mlx::last_dim;
using gsplat_b200_mlx::out_ptr;
using gsplat_b200_mlx::ptr;

// ------------------------------------------------ quat/scale -> covariance

// Replaces gsplat_quat_scale_to_covar.cpp:471-511 (Metal dispatch).
void GSPlatQuatScaleToCovarPreci::eval_gpu(const std::vector<mx::array>& inputs,
                                           std::vector<mx::array>& outputs) {
  allocate(outputs);
  const int64_t n = static_cast<int64_t>(inputs[0].size() / 4);
  if (n == 0) {
    return;
  }
  gs_qs2c_params p{n, compute_covar_, compute_preci_, triu_};
  Launch L(stream());
  L.done(gs_quat_scale_to_covar_fwd(&p, inputs[0].data<float>(), inputs[1].data<float>(),
                                    compute_covar_ ? outputs[kCovars].data<float>() : nullptr,
                                    compute_preci_ ? outputs[kPrecis].data<float>() : nullptr,
                                    L.stream()),
         "quat_scale_to_covar_preci_forward");
}

// Replaces gsplat_quat_scale_to_covar.cpp:513-558.
void GSPlatQuatScaleToCovarPreciBackward::eval_gpu(const std::vector<mx::array>& inputs,
                                                   std::vector<mx::array>& outputs) {
  allocate(outputs);
  const int64_t n = static_cast<int64_t>(inputs[0].size() / 4);
  if (n == 0) {
    return;
  }
  gs_qs2c_params p{n, use_v_covars_, use_v_precis_, triu_};
  Launch L(stream());
  L.done(gs_quat_scale_to_covar_bwd(&p, inputs[0].data<float>(), inputs[1].data<float>(),
                                    use_v_covars_ ? inputs[2].data<float>() : nullptr,
                                    use_v_precis_ ? inputs[3].data<float>() : nullptr,
                                    outputs[0].data<float>(), outputs[1].data<float>(),
                                    L.stream()),
         "quat_scale_to_covar_preci_backward");
}

// ------------------------------------------------------------- projection

namespace {

gs_projection_params projection_params(const ProjectionEWA3DGSFusedParams& q,
                                       const mx::array& means, const mx::array& viewmats) {
  gs_projection_params p{};
  p.N = last_dim(means, 2);
  p.C = last_dim(viewmats, 3);
  p.B = p.N == 0 ? 0 : static_cast<int32_t>(means.size() / (static_cast<size_t>(p.N) * 3));
  p.image_width = q.image_width;
  p.image_height = q.image_height;
  p.eps2d = q.eps2d;
  p.near_plane = q.near_plane;
  p.far_plane = q.far_plane;
  p.radius_clip = q.radius_clip;
  p.calc_compensations = q.calc_compensations;
  p.camera_model = q.camera_model;
  p.use_covars = q.use_covars;
  p.use_opacities = q.use_opacities;
  return p;
}

}  // namespace

// Replaces gsplat_projection.cpp:655-737 (Metal dispatch of the forward).
void GSPlatProjectionEWA3DGSFused::eval_gpu(const std::vector<mx::array>& inputs,
                                            std::vector<mx::array>& outputs) {
  allocate(outputs);
  const auto& means = inputs[0];
  const auto& viewmats = inputs[5];
  gs_projection_params p = projection_params(params_, means, viewmats);
  if (static_cast<int64_t>(p.B) * p.C * p.N == 0) {
    return;
  }
  Launch L(stream());
  L.done(gs_projection_fwd(
             &p, means.data<float>(), params_.use_covars ? inputs[1].data<float>() : nullptr,
             params_.use_covars ? nullptr : inputs[2].data<float>(),
             params_.use_covars ? nullptr : inputs[3].data<float>(),
             params_.use_opacities ? inputs[4].data<float>() : nullptr, viewmats.data<float>(),
             inputs[6].data<float>(), outputs[kMeans2D].data<float>(),
             outputs[kDepths].data<float>(), outputs[kConics].data<float>(),
             params_.calc_compensations ? outputs[kCompensations].data<float>() : nullptr,
             outputs[kRadii].data<int32_t>(), L.stream()),
         "projection_ewa_3dgs_fused_forward");
}

// Replaces gsplat_projection.cpp:739-855 (Metal dispatch of the backward,
// including its v_viewmats pass when viewmats_requires_grad).
void GSPlatProjectionEWA3DGSFusedBackward::eval_gpu(const std::vector<mx::array>& inputs,
                                                    std::vector<mx::array>& outputs) {
  allocate(outputs);
  const auto& means = inputs[0];
  const auto& viewmats = inputs[4];
  gs_projection_params p = projection_params(params_, means, viewmats);
  if (static_cast<int64_t>(p.B) * p.N == 0) {
    // the reference returns before its zero-fill's only consumer; the
    // outputs still get defined zeros here
    for (auto& out : outputs) {
      if (out.nbytes() != 0) {
        std::memset(out.data<void>(), 0, out.nbytes());
      }
    }
    return;
  }
  const bool comp = params_.calc_compensations;
  Launch L(stream());
  L.done(gs_projection_bwd(
             &p, means.data<float>(), params_.use_covars ? inputs[1].data<float>() : nullptr,
             params_.use_covars ? nullptr : inputs[2].data<float>(),
             params_.use_covars ? nullptr : inputs[3].data<float>(), viewmats.data<float>(),
             inputs[5].data<float>(), inputs[6].data<int32_t>(), inputs[7].data<float>(),
             comp ? ptr<float>(inputs[8]) : nullptr, inputs[9].data<float>(),
             inputs[10].data<float>(), inputs[11].data<float>(),
             comp ? ptr<float>(inputs[12]) : nullptr,
             outputs[kProjectionVMeans].data<float>(),
             out_ptr<float>(outputs[kProjectionVCovars]),
             out_ptr<float>(outputs[kProjectionVQuats]),
             out_ptr<float>(outputs[kProjectionVScales]),
             viewmats_requires_grad_ ? outputs[kProjectionVViewmats].data<float>() : nullptr,
             L.stream()),
         "projection_ewa_3dgs_fused_backward");
}

// ---------------------------------------------------- spherical harmonics

// Replaces gsplat_spherical_harmonics.cpp:557-598.
void GSPlatSphericalHarmonics::eval_gpu(const std::vector<mx::array>& inputs,
                                        std::vector<mx::array>& outputs) {
  allocate(outputs);
  const auto& dirs = inputs[0];
  const auto& coeffs = inputs[1];
  gs_sh_params p{static_cast<int64_t>(dirs.size() / 3), last_dim(coeffs, 2), degrees_to_use_,
                 use_masks_};
  if (p.n == 0) {
    return;
  }
  Launch L(stream());
  L.done(gs_sh_fwd(&p, dirs.data<float>(), coeffs.data<float>(),
                   use_masks_ ? inputs[2].data<uint8_t>() : nullptr, outputs[0].data<float>(),
                   L.stream()),
         "spherical_harmonics_forward");
}

// Replaces gsplat_spherical_harmonics.cpp:600-646.
void GSPlatSphericalHarmonicsBackward::eval_gpu(const std::vector<mx::array>& inputs,
                                                std::vector<mx::array>& outputs) {
  allocate(outputs);
  const auto& dirs = inputs[0];
  const auto& coeffs = inputs[1];
  gs_sh_params p{static_cast<int64_t>(dirs.size() / 3), last_dim(coeffs, 2), degrees_to_use_,
                 use_masks_};
  if (p.n == 0) {
    return;
  }
  Launch L(stream());
  L.done(gs_sh_bwd(&p, dirs.data<float>(), coeffs.data<float>(),
                   use_masks_ ? inputs[2].data<uint8_t>() : nullptr, inputs[3].data<float>(),
                   compute_v_dirs_ ? outputs[kSHVDirs].data<float>() : nullptr,
                   outputs[kSHVCoeffs].data<float>(), L.stream()),
         "spherical_harmonics_backward");
}

// ---------------------------------------------------------------- intersect

namespace {

gs_isect_params isect_params(int I, int tile_size, int tile_width, int tile_height,
                             const mx::array& depths) {
  gs_isect_params p{};
  p.I = I;
  p.N = I > 0 ? static_cast<int32_t>(depths.size() / static_cast<size_t>(I)) : 0;
  p.tile_size = tile_size;
  p.tile_width = tile_width;
  p.tile_height = tile_height;
  return p;
}

}  // namespace

// Replaces gsplat_intersect.cpp:342-382.
void GSPlatIntersectTileCount::eval_gpu(const std::vector<mx::array>& inputs,
                                        std::vector<mx::array>& outputs) {
  allocate(outputs);
  const auto& depths = inputs[2];
  if (depths.size() == 0) {
    return;
  }
  gs_isect_params p = isect_params(params_.I, params_.tile_size, params_.tile_width,
                                   params_.tile_height, depths);
  Launch L(stream());
  L.done(gs_isect_tile_count(&p, inputs[0].data<float>(), inputs[1].data<int32_t>(),
                             outputs[0].data<int32_t>(), L.stream()),
         "intersect_tile_count");
}

// Replaces gsplat_intersect.cpp:488-539: the intersections in the
// reference's encode order (element order, then tile rows / columns).
void GSPlatIntersectTileEncode::eval_gpu(const std::vector<mx::array>& inputs,
                                         std::vector<mx::array>& outputs) {
  allocate(outputs);
  const auto& depths = inputs[2];
  const int64_t n_isects = params_.total_isects;
  if (depths.size() == 0 || n_isects == 0) {
    return;
  }
  gs_isect_params p = isect_params(params_.I, params_.tile_size, params_.tile_width,
                                   params_.tile_height, depths);
  Launch L(stream());
  L.done(gs_isect_tile_encode(&p, inputs[0].data<float>(), inputs[1].data<int32_t>(),
                              depths.data<float>(), inputs[3].data<int32_t>(), n_isects,
                              outputs[0].data<int64_t>(), outputs[1].data<int32_t>(),
                              L.stream()),
         "intersect_tile_encode");
}

// Replaces gsplat_intersect.cpp:644-681.
void GSPlatIntersectOffset::eval_gpu(const std::vector<mx::array>& inputs,
                                     std::vector<mx::array>& outputs) {
  allocate(outputs);
  if (outputs[0].size() == 0) {
    return;
  }
  Launch L(stream());
  L.done(gs_isect_offset(static_cast<int64_t>(inputs[0].size()), ptr<int64_t>(inputs[0]),
                         params_.I, params_.tile_width, params_.tile_height,
                         outputs[0].data<int32_t>(), L.stream()),
         "intersect_offset");
}

// ---------------------------------------------------------------- rasterize

namespace {

gs_raster_params raster_params(const RasterizeToPixels3DGSParams& q,
                               const std::vector<mx::array>& inputs) {
  const auto& means2d = inputs[0];
  const auto& colors = inputs[2];
  const auto& tile_offsets = inputs[6];
  const int th = last_dim(tile_offsets, 2);
  const int tw = last_dim(tile_offsets, 1);
  gs_raster_params p{};
  const size_t n_tiles = static_cast<size_t>(th) * static_cast<size_t>(tw);
  p.I = n_tiles == 0 ? 0 : static_cast<int32_t>(tile_offsets.size() / n_tiles);
  p.N = last_dim(means2d, 2);
  p.channels = last_dim(colors, 1);
  p.image_width = q.image_width;
  p.image_height = q.image_height;
  p.tile_size = q.tile_size;
  p.tile_width = tw;
  p.tile_height = th;
  p.n_isects = static_cast<int64_t>(inputs[7].size());
  p.use_backgrounds = q.use_backgrounds;
  p.use_masks = q.use_masks;
  return p;
}

}  // namespace

// Replaces gsplat_rasterize.cpp:572-641.
void GSPlatRasterizeToPixels3DGS::eval_gpu(const std::vector<mx::array>& inputs,
                                           std::vector<mx::array>& outputs) {
  allocate(outputs);
  if (outputs[kLastIds].size() == 0) {
    return;
  }
  gs_raster_params p = raster_params(params_, inputs);
  Launch L(stream());
  L.done(gs_rasterize_fwd(&p, inputs[0].data<float>(), inputs[1].data<float>(),
                          inputs[2].data<float>(), inputs[3].data<float>(),
                          params_.use_backgrounds ? inputs[4].data<float>() : nullptr,
                          params_.use_masks ? inputs[5].data<uint8_t>() : nullptr,
                          inputs[6].data<int32_t>(), ptr<int32_t>(inputs[7]),
                          outputs[kRenderColors].data<float>(),
                          outputs[kRenderAlphas].data<float>(),
                          outputs[kLastIds].data<int32_t>(), L.stream()),
         "rasterize_to_pixels_3dgs_forward");
}

// Replaces gsplat_rasterize.cpp:643-724.
void GSPlatRasterizeToPixels3DGSBackward::eval_gpu(const std::vector<mx::array>& inputs,
                                                   std::vector<mx::array>& outputs) {
  allocate(outputs);
  if (inputs[8].size() == 0) {
    for (auto& out : outputs) {
      if (out.nbytes() != 0) {
        std::memset(out.data<void>(), 0, out.nbytes());
      }
    }
    return;
  }
  gs_raster_params p = raster_params(params_, inputs);
  p.absgrad = absgrad_;
  Launch L(stream());
  L.done(gs_rasterize_bwd(&p, inputs[0].data<float>(), inputs[1].data<float>(),
                          inputs[2].data<float>(), inputs[3].data<float>(),
                          params_.use_backgrounds ? inputs[4].data<float>() : nullptr,
                          params_.use_masks ? inputs[5].data<uint8_t>() : nullptr,
                          inputs[6].data<int32_t>(), ptr<int32_t>(inputs[7]),
                          inputs[8].data<float>(), inputs[9].data<int32_t>(),
                          inputs[10].data<float>(), inputs[11].data<float>(),
                          absgrad_ ? outputs[kRasterVMeans2DAbs].data<float>() : nullptr,
                          outputs[kRasterVMeans2D].data<float>(),
                          outputs[kRasterVConics].data<float>(),
                          outputs[kRasterVColors].data<float>(),
                          outputs[kRasterVOpacities].data<float>(),
                          params_.use_backgrounds ? outputs[kRasterVBackgrounds].data<float>()
                                                  : nullptr,
                          L.stream()),
         "rasterize_to_pixels_3dgs_backward");
}

}  // namespace gsplat_core
