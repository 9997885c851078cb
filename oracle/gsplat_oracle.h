/*
 * CPU oracle for the gsplat_core hot path: a plain-C restatement of the
 * reference operators' CPU algorithms (gsplat-mlx, gsplat_core/gsplat_{op}.cpp
 * `eval_cpu` bodies; the projection forward follows the Metal `eval_gpu`
 * culling rules, gsplat_core/metal/gsplat_projection.metal:249-326).
 *
 * TEST INFRASTRUCTURE ONLY.  It is the checker for the CUDA kernels and the
 * timed CPU baseline ("port").  Only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline leg may load it; the product never does.
 *
 * Parity pinning: tests/test_oracle_golden.py checks every function here
 * against the tests/golden fixtures, which tests/golden/make_golden.py produced by
 * running the reference's own eval_cpu code (oracle/_ref) and the known
 * answers of gsplat_core/test/test.cpp.
 *
 * Layouts are the reference's dense layouts, row-major, float32 unless
 * noted.  All functions return 0 on success, a negative value on invalid
 * arguments.
 */
#ifndef GSPLAT_ORACLE_H
#define GSPLAT_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

int orc_qs2c_fwd(int64_t n, const float* quats, const float* scales,
                 int compute_covar, int compute_preci, int triu, float* covars,
                 float* precis);
int orc_qs2c_bwd(int64_t n, const float* quats, const float* scales,
                 const float* v_covars, const float* v_precis, int triu,
                 float* v_quats, float* v_scales);

int orc_proj_fwd(int B, int C, int N, const float* means, const float* covars,
                 const float* quats, const float* scales,
                 const float* opacities, const float* viewmats, const float* Ks,
                 int width, int height, float eps2d, float near_plane,
                 float far_plane, float radius_clip, int calc_compensations,
                 int camera_model, float* means2d, float* depths,
                 float* conics, float* compensations, int32_t* radii);
int orc_proj_bwd(int B, int C, int N, const float* means, const float* covars,
                 const float* quats, const float* scales,
                 const float* viewmats, const float* Ks, int width, int height,
                 float eps2d, const int32_t* radii, const float* conics,
                 const float* compensations, const float* v_means2d,
                 const float* v_depths, const float* v_conics,
                 const float* v_compensations, float* v_means,
                 float* v_covars, float* v_quats, float* v_scales,
                 float* v_viewmats);

int orc_sh_fwd(int64_t n, int K, int degree, const float* dirs,
               const float* coeffs, const uint8_t* masks, float* colors);
int orc_sh_bwd(int64_t n, int K, int degree, const float* dirs,
               const float* coeffs, const uint8_t* masks,
               const float* v_colors, float* v_dirs, float* v_coeffs);

int orc_isect_count(int I, int N, const float* means2d, const int32_t* radii,
                    int tile_size, int tile_width, int tile_height,
                    int32_t* tiles_per_gauss);
int64_t orc_isect_scan(int64_t n, const int32_t* counts, int32_t* offsets);
int orc_isect_encode(int I, int N, const float* means2d, const int32_t* radii,
                     const float* depths, const int32_t* offsets,
                     int tile_size, int tile_width, int tile_height,
                     int64_t n_isects, int64_t* isect_ids,
                     int32_t* flatten_ids);
int orc_isect_sort(int64_t n_isects, const int64_t* isect_ids,
                   const int32_t* flatten_ids, int64_t* sorted_ids,
                   int32_t* sorted_flatten);
int orc_isect_offset(int64_t n_isects, const int64_t* isect_ids, int I,
                     int tile_width, int tile_height, int32_t* offsets);

int orc_raster_fwd(int I, int N, int channels, const float* means2d,
                   const float* conics, const float* colors,
                   const float* opacities, const float* backgrounds,
                   const uint8_t* masks, int width, int height, int tile_size,
                   int tile_width, int tile_height, const int32_t* tile_offsets,
                   int64_t n_isects, const int32_t* flatten_ids,
                   float* render_colors, float* render_alphas,
                   int32_t* last_ids, int nthreads);
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
                   int nthreads);

int orc_sh_glue_fwd(int C, int N, int K, int degree, const float* means,
                    const float* viewmats, const float* coeffs,
                    const uint8_t* masks, float* colors);
int orc_sh_glue_bwd(int C, int N, int K, int degree, const float* means,
                    const float* viewmats, const float* coeffs,
                    const uint8_t* masks, const float* v_colors_out,
                    float* v_means, float* v_coeffs);

#ifdef __cplusplus
}
#endif

#endif
