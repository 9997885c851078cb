/*
 * gsplat_b200 -- C ABI of the B200 (sm_100a) implementation of gsplat-mlx's
 * five differentiable 3D Gaussian Splatting operators.
 *
 * Every entry point:
 *   - takes raw DEVICE pointers (float32 / int32 / int64 / uint8-as-bool,
 *     dense row-major, the reference's layouts), a pointer to a POD
 *     parameter struct and a CUDA stream (cudaStream_t passed as void*);
 *   - enqueues its kernels on that stream and returns without waiting;
 *   - writes every element of every output it is given (the reference
 *     zero-fills its outputs before eval, e.g. gsplat_rasterize.cpp:575-578;
 *     here culled / masked entries are written as exact zeros on device);
 *   - never allocates device memory: scratch is passed in by the caller as a
 *     workspace whose size the matching *_workspace_size() function returns;
 *   - returns GS_OK or an error status; gs_last_error() then holds a message
 *     (thread-local).  Invalid shapes / sizes are rejected before any launch,
 *     as the reference's front-ends throw std::runtime_error
 *     (e.g. gsplat_projection.cpp:115-141).
 *
 * Each function names the reference interface it replaces (file:line inside
 * the gsplat-mlx repository).  In the reference, the Metal dispatch blocks of
 * the Primitive::eval_gpu methods are the call sites these entries replace.
 */
#ifndef GSPLAT_B200_H
#define GSPLAT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void* gs_stream_t; /* a cudaStream_t; NULL is the legacy stream */

enum gs_status {
  GS_OK = 0,
  GS_ERR_INVALID = 1,     /* bad shape / argument (reference: runtime_error) */
  GS_ERR_UNSUPPORTED = 2, /* path the reference also rejects (packed, ...)   */
  GS_ERR_OVERFLOW = 3,    /* int32 index limits of the operator surface      */
  GS_ERR_CUDA = 4,        /* a CUDA launch / runtime error                   */
  GS_ERR_WORKSPACE = 5,   /* workspace pointer missing or too small          */
  GS_ERR_DEVICE = 6       /* a kernel reported a failed on-device check      */
};

const char* gs_status_string(int status);
const char* gs_last_error(void);
int gs_version(void); /* major*10000 + minor*100 + patch */

/* ------------------------------------------------------------------ */
/* quat/scale -> covariance / precision                                */
/* Replaces GSPlatQuatScaleToCovarPreci{,Backward}::eval_gpu,          */
/* gsplat_quat_scale_to_covar.cpp:471-558; params mirror               */
/* QuatScaleToCovarPreciKernelParams, :27-32.                          */
/* ------------------------------------------------------------------ */
typedef struct {
  int64_t n;             /* number of (quat, scale) pairs                */
  int32_t compute_covar; /* fwd: write covars; bwd: v_covars is given    */
  int32_t compute_preci; /* fwd: write precis; bwd: v_precis is given    */
  int32_t triu;          /* 1: [n,6] upper triangle; 0: [n,3,3]          */
} gs_qs2c_params;

int gs_quat_scale_to_covar_fwd(const gs_qs2c_params* p, const float* quats,
                               const float* scales, float* covars,
                               float* precis, gs_stream_t stream);
int gs_quat_scale_to_covar_bwd(const gs_qs2c_params* p, const float* quats,
                               const float* scales, const float* v_covars,
                               const float* v_precis, float* v_quats,
                               float* v_scales, gs_stream_t stream);

/* ------------------------------------------------------------------ */
/* fully fused EWA projection                                          */
/* Replaces GSPlatProjectionEWA3DGSFused{,Backward}::eval_gpu,         */
/* gsplat_projection.cpp:655-855; params mirror ProjectionKernelParams */
/* (:26-40) and ProjectionEWA3DGSFusedParams (gsplat_projection.h:12). */
/* ------------------------------------------------------------------ */
typedef struct {
  int32_t B, C, N;
  int32_t image_width, image_height;
  float eps2d, near_plane, far_plane, radius_clip;
  int32_t calc_compensations;
  int32_t camera_model; /* 0 pinhole, 1 orthographic, 2 fisheye (fwd only) */
  int32_t use_covars;   /* 1: covars [B,N,6]; 0: quats [B,N,4] + scales    */
  int32_t use_opacities;
} gs_projection_params;

/* Outputs: means2d [B,C,N,2], depths [B,C,N], conics [B,C,N,3],
 * compensations [B,C,N] (only when calc_compensations), radii [B,C,N,2]. */
int gs_projection_fwd(const gs_projection_params* p, const float* means,
                      const float* covars, const float* quats,
                      const float* scales, const float* opacities,
                      const float* viewmats, const float* Ks, float* means2d,
                      float* depths, float* conics, float* compensations,
                      int32_t* radii, gs_stream_t stream);
/* v_viewmats may be NULL (reference: viewmats_requires_grad == false).
 * v_compensations may be NULL; it is read only when calc_compensations. */
int gs_projection_bwd(const gs_projection_params* p, const float* means,
                      const float* covars, const float* quats,
                      const float* scales, const float* viewmats,
                      const float* Ks, const int32_t* radii,
                      const float* conics, const float* compensations,
                      const float* v_means2d, const float* v_depths,
                      const float* v_conics, const float* v_compensations,
                      float* v_means, float* v_covars, float* v_quats,
                      float* v_scales, float* v_viewmats, gs_stream_t stream);

/* ------------------------------------------------------------------ */
/* spherical harmonics, degree 0..4                                    */
/* Replaces GSPlatSphericalHarmonics{,Backward}::eval_gpu,             */
/* gsplat_spherical_harmonics.cpp:557-646; params mirror               */
/* SphericalHarmonicsKernelParams, :26-31.                             */
/* ------------------------------------------------------------------ */
typedef struct {
  int64_t n;              /* prod(dirs.shape[:-1])                        */
  int32_t K;              /* coeffs.shape[-2] (>= (degree+1)^2)           */
  int32_t degrees_to_use; /* 0..4                                         */
  int32_t use_masks;      /* masks [n] uint8 given                        */
} gs_sh_params;

int gs_sh_fwd(const gs_sh_params* p, const float* dirs, const float* coeffs,
              const uint8_t* masks, float* colors, gs_stream_t stream);
/* v_dirs may be NULL (reference: compute_v_dirs == false). */
int gs_sh_bwd(const gs_sh_params* p, const float* dirs, const float* coeffs,
              const uint8_t* masks, const float* v_colors, float* v_dirs,
              float* v_coeffs, gs_stream_t stream);

/* Fused SH colour glue of the reference trainers
 * (scripts/test/scanner_points_training_utils.py:1005-1034):
 *   colors[c,n] = clip(SH(normalize(means[n] - campos_c), coeffs[n]) + 0.5, 0, 1)
 * with campos_c = -R_c^T t_c.  Entries can be skipped: by masks [C,N]
 * (uint8, optional) and/or by radii [C,N,2] (int32, optional; an entry is
 * visible when both radii are > 0, the projection's culling result).  A
 * skipped entry gets colour 0 and no gradient -- the rasterizer never reads
 * the colour of a culled Gaussian, so the rendered image and every gradient
 * are unchanged.  The backward adds the reverse mode of the composition
 * (clip masks, SH, normalisation) into v_means [N,3] and writes v_coeffs
 * [N,K,3] summed over the C cameras.  */
typedef struct {
  int32_t C, N, K, degrees_to_use;
  int32_t use_masks;
  int32_t skip_zero_cotangents; /* bwd: an entry whose colour cotangent is 0
                                   contributes nothing and is skipped (for
                                   cameras whose radii are not at hand) */
  int32_t camera_groups; /* bwd: > 1 = the colour cotangents (and masks /
                            radii) come in the order of G = camera_groups
                            groups interleaved: entry camera c = j G + g is
                            camera j of group g, whose pose is viewmats row
                            g (C / G) + j (the order a camera-sharded step's
                            per-camera all-to-alls deliver them); else the
                            viewmats order */
} gs_sh_glue_params;

int gs_sh_glue_fwd(const gs_sh_glue_params* p, const float* means,
                   const float* viewmats, const float* coeffs,
                   const uint8_t* masks, const int32_t* radii, float* colors,
                   gs_stream_t stream);
int gs_sh_glue_bwd(const gs_sh_glue_params* p, const float* means,
                   const float* viewmats, const float* coeffs,
                   const uint8_t* masks, const int32_t* radii,
                   const float* v_colors, float* v_means_accum,
                   float* v_coeffs, gs_stream_t stream);

/* ------------------------------------------------------------------ */
/* tile intersection                                                   */
/* Replaces GSPlatIntersectTileCount / GSPlatIntersectTileEncode /     */
/* GSPlatIntersectOffset ::eval_gpu (gsplat_intersect.cpp:342-382,     */
/* :488-539, :644-681), MLX cumsum in gsplat_intersect_tile_offsets    */
/* (:196-211) and MLX argsort+take in gsplat_intersect_tile_sort       */
/* (:266-286).  Params mirror IntersectTileCountKernelParams /         */
/* IntersectTileEncodeKernelParams (:29-51).                           */
/* ------------------------------------------------------------------ */
typedef struct {
  int32_t I;          /* images (B*C)                                    */
  int32_t N;          /* Gaussians per image                             */
  int32_t tile_size, tile_width, tile_height;
  int32_t tile_y0, tile_y1; /* when tile_y1 > tile_y0: only tile rows
                               [tile_y0, tile_y1) are intersected (a band of
                               the image; keys keep absolute tile ids); else
                               all rows, as the reference */
  int32_t reuse_depth_order; /* gs_isect_tile_encode_sorted: 1 = the
                                workspace holds the depth order of an earlier
                                call with the same I, N, radii and depths (the
                                other bands of a step); its element sort is
                                skipped */
  int32_t positive_depths;   /* gs_isect_tile_encode_binned: 1 = the caller
                                promises that every element with positive
                                radii has a depth with the sign bit clear
                                (a projection with near_plane > 0 gives
                                that); the sort then carries 31 depth bits,
                                one key bit fewer.  Same output; a broken
                                promise misorders, it does not fault. */
  int32_t shared_opacities;  /* gs_isect_tile_encode_binned_culled: 1 =
                                opacities are [N], shared by the I images
                                (element e reads e mod N); else [I, N] */
} gs_isect_params;

/* tiles_per_gauss [I,N] int32 */
int gs_isect_tile_count(const gs_isect_params* p, const float* means2d,
                        const int32_t* radii, int32_t* tiles_per_gauss,
                        gs_stream_t stream);
/* The same counts and, in one pass, their total into a device int64 (the
 * total that gs_isect_scan also produces), for callers that need only the
 * total before the sorted encode.  No reference counterpart. */
int gs_isect_tile_count_total(const gs_isect_params* p, const float* means2d,
                              const int32_t* radii, int32_t* tiles_per_gauss,
                              int64_t* total_device, gs_stream_t stream);

/* Exclusive prefix sum of n int32 counts into offsets (int32, as the
 * reference's cumsum), and the 64-bit total into *total_device (a device
 * int64).  Totals of 2^31 or more are an overflow of the reference's int32
 * offsets; the caller checks *total_device. */
size_t gs_isect_scan_workspace_size(int64_t n);
int gs_isect_scan(int64_t n, const int32_t* counts, int32_t* offsets,
                  int64_t* total_device, void* workspace,
                  size_t workspace_bytes, gs_stream_t stream);

/* isect_ids [n_isects] int64 (image|tile|depth bits), flatten_ids int32 */
int gs_isect_tile_encode(const gs_isect_params* p, const float* means2d,
                         const int32_t* radii, const float* depths,
                         const int32_t* offsets, int64_t n_isects,
                         int64_t* isect_ids, int32_t* flatten_ids,
                         gs_stream_t stream);

/* Encode and sort in one call: the output equals gs_isect_tile_encode
 * followed by gs_isect_sort over all key bits (the reference's encode +
 * mx::argsort + 2x mx::take, gsplat_intersect.cpp:266-286 and :488-539,
 * i.e. isect_tiles with sort=True), bit for bit.  Inside, the I*N elements
 * are first ordered by their depth bits, the intersections are encoded in
 * that order, and only the tile and image bits are sorted afterwards.
 * tiles_per_gauss [I*N] comes from gs_isect_tile_count; n_isects is its
 * total.  The workspace is sized by
 * gs_isect_tile_encode_sorted_workspace_size(I*N, n_isects). */
size_t gs_isect_tile_encode_sorted_workspace_size(int64_t n_elements, int64_t n_isects);
int gs_isect_tile_encode_sorted(const gs_isect_params* p, const float* means2d,
                                const int32_t* radii, const float* depths,
                                const int32_t* tiles_per_gauss, int64_t n_isects,
                                int64_t* isect_ids, int32_t* flatten_ids,
                                void* workspace, size_t workspace_bytes,
                                gs_stream_t stream);

/* Binned encode and sort: the same isect_ids / flatten_ids as
 * gs_isect_tile_encode_sorted (bit for bit the reference's sorted encode),
 * built another way: every element lists itself once per 4x4-tile bin its
 * tile rect touches, those entries are sorted by (bin, depth bits), and one
 * CTA per tile keeps, in that order, the elements of its bin that cover it.
 * With tile_offsets (the [I, rows, tile_width] slots of the call's tile
 * rows, else NULL) it also writes what gs_isect_offset_rows would.
 * n_isects and n_bin_entries are the two totals of
 * gs_isect_tile_count_totals over the same rows; the workspace is sized by
 * gs_isect_tile_encode_binned_workspace_size(p, n_bin_entries).  Tile grids
 * wider or taller than 65535 tiles are refused (GS_ERR_INVALID).
 * No reference counterpart. */
/* Copies n (<= 1024) int64 from device memory into pinned host memory with a
 * kernel's stores through the buffer's device mapping, so that a host read of
 * a few totals (the intersection count of a step) does not wait on the copy
 * engines behind another stream's large download; without a mapping it is a
 * cudaMemcpyAsync.  The values are on the host once `stream` has passed this
 * point.  No reference counterpart (the reference reads its total with
 * MLX's item()). */
int gs_store_to_host_i64(const int64_t* src, int64_t* host_dst, int32_t n,
                         gs_stream_t stream);
int gs_isect_tile_count_totals(const gs_isect_params* p, const float* means2d,
                               const int32_t* radii, int32_t* tiles_per_gauss,
                               int64_t* totals_device /* [2]: intersections, bin entries */,
                               gs_stream_t stream);
size_t gs_isect_tile_encode_binned_workspace_size(const gs_isect_params* p,
                                                  int64_t n_bin_entries);
int gs_isect_tile_encode_binned(const gs_isect_params* p, const float* means2d,
                                const int32_t* radii, const float* depths,
                                int64_t n_isects, int64_t n_bin_entries,
                                int64_t* isect_ids, int32_t* flatten_ids,
                                int32_t* tile_offsets, void* workspace,
                                size_t workspace_bytes, gs_stream_t stream);

/* Opacity-aware tile culling on top of the binned encode: the tile lists
 * of gs_isect_tile_encode_binned with every (tile, element) pair removed
 * for which the element's opacity-weighted Gaussian (conics [I,N,3],
 * opacities [I,N], the rasterizer's inputs) stays below alpha 1/255 at
 * every pixel centre of the tile, by a margin that covers fp32 rounding.
 * The rasterizer skips such a pair at every pixel, so rendering the culled
 * lists gives the same colours and alphas bit for bit; only the list
 * positions (and so last_ids) change.  The kept lists keep their order and
 * fill the LAST n_kept places of isect_ids / flatten_ids [n_isects]:
 * tile_offsets point there, so that the last tile still ends at n_isects
 * and a rasterizer call with the same n_isects needs no host read.
 * *n_kept (device int64, may be NULL) receives the kept total.  Same
 * workspace as gs_isect_tile_encode_binned.
 * Replaces the conics / opacities arguments of intersect_tile_forward,
 * which the reference accepts and refuses (gsplat_intersect.cpp:115-126). */
int gs_isect_tile_encode_binned_culled(const gs_isect_params* p, const float* means2d,
                                       const int32_t* radii, const float* depths,
                                       const float* conics, const float* opacities,
                                       int64_t n_isects, int64_t n_bin_entries,
                                       int64_t* isect_ids, int32_t* flatten_ids,
                                       int32_t* tile_offsets, int64_t* n_kept,
                                       void* workspace, size_t workspace_bytes,
                                       gs_stream_t stream);

/* Packed [nnz] layout -- the upstream-gsplat form the reference refuses
 * ("intersect_tile packed path is not implemented yet",
 * gsplat_intersect.cpp:115-118, image_ids / gaussian_ids inputs of
 * intersect_tile_forward).
 *
 * gs_pack_visible: the visible (both radii > 0) entries of a dense
 * projection output [n_elements = I*N] as rows in (image, Gaussian) order:
 * image_ids, gaussian_ids [nnz], radii [nnz,2], means2d [nnz,2], depths
 * [nnz], conics [nnz,3], compensations [nnz] (when given).  *nnz_device gets
 * the row count; rows past `capacity` are not written (size the outputs
 * with a first call of capacity 0, or with an upper bound).  Workspace:
 * gs_pack_visible_workspace_size(n_elements) bytes.
 *
 * gs_isect_tile_encode_binned_packed: the binned encode over nnz packed
 * rows (p->N = nnz, p->I = images): element i's image is image_ids[i],
 * which must lie in [0, I); flatten_ids are row indices.  n_isects /
 * n_bin_entries come from gs_isect_tile_count_totals over the rows (I = 1,
 * N = nnz: the counts do not depend on the image).  The rasterizer entries
 * render packed rows as they are (pass N = 0 so that they do not size
 * anything by I * N, and zero the gradient buffers first). */
size_t gs_pack_visible_workspace_size(int64_t n_elements);
int gs_pack_visible(int64_t n_elements, int32_t N, const int32_t* radii,
                    const float* means2d, const float* depths,
                    const float* conics, const float* compensations,
                    int64_t capacity, int32_t* image_ids, int32_t* gaussian_ids,
                    int32_t* p_radii, float* p_means2d, float* p_depths,
                    float* p_conics, float* p_compensations,
                    int64_t* nnz_device, void* workspace, size_t workspace_bytes,
                    gs_stream_t stream);
size_t gs_isect_tile_encode_binned_packed_workspace_size(const gs_isect_params* p,
                                                         int64_t n_bin_entries);
int gs_isect_tile_encode_binned_packed(const gs_isect_params* p,
                                       const int32_t* image_ids,
                                       const float* means2d, const int32_t* radii,
                                       const float* depths, int64_t n_isects,
                                       int64_t n_bin_entries, int64_t* isect_ids,
                                       int32_t* flatten_ids, int32_t* tile_offsets,
                                       void* workspace, size_t workspace_bytes,
                                       gs_stream_t stream);

/* The radix passes of the calls above and below wait on one another's
 * tiles with bounded waits; a wait that gives up (a defect, not a workload
 * condition) raises an error word in the workspace and the kernels finish
 * with invalid output.  These read that word for the last call that used
 * the workspace: they wait for `stream`, then return GS_OK or GS_ERR_DEVICE.
 * No reference counterpart. */
int gs_isect_tile_encode_sorted_check(int64_t n_elements, int64_t n_isects,
                                      const void* workspace, gs_stream_t stream);
int gs_isect_tile_encode_binned_check(int64_t n_bin_entries, const void* workspace,
                                      gs_stream_t stream);
int gs_isect_sort_check(int64_t n_isects, const void* workspace, gs_stream_t stream);

/* Stable ascending sort of (isect_ids, flatten_ids) by the signed 64-bit
 * key, equal keys kept in input order -- the result of MLX's argsort+take.
 * key_bits = 32 + tile_bits + image_bits is the number of low key bits
 * that can be non-zero (the rest must be zero); 1..64.  */
size_t gs_isect_sort_workspace_size(int64_t n_isects);
int gs_isect_sort(int64_t n_isects, int32_t key_bits, const int64_t* isect_ids,
                  const int32_t* flatten_ids, int64_t* sorted_isect_ids,
                  int32_t* sorted_flatten_ids, void* workspace,
                  size_t workspace_bytes, gs_stream_t stream);

/* The same stable sort for callers that may not allocate device memory while
 * they run (for example a host engine that owns every device buffer and gives
 * plugins only their inputs and outputs).  It has no counterpart in the
 * reference.  Its scratch is a fixed 13 MiB array inside this library, held
 * on every GPU that loads the library until the process exits; it sorts at
 * most 1,048,576 intersections and returns GS_ERR_INVALID for more, before
 * launching anything.  It calls no allocator.  The first call on a device
 * looks the array's device address up (cudaGetSymbolAddress) with that device
 * current -- make that first call before any stream capture.  All calls share
 * the one array, which keeps the last call's contents: calls that may overlap
 * on the GPU (several streams, several host threads) race and must be
 * serialised by the caller. */
int gs_isect_sort_noalloc(int64_t n_isects, int32_t key_bits,
                          const int64_t* isect_ids, const int32_t* flatten_ids,
                          int64_t* sorted_isect_ids, int32_t* sorted_flatten_ids,
                          gs_stream_t stream);
/* The error word of the last gs_isect_sort_noalloc call on the current
 * device (n_isects as passed to it), read from the library's fixed array:
 * waits for `stream`, then GS_OK, or GS_ERR_DEVICE when a bounded wait of
 * that sort gave up.  GS_OK before the first call.  The array's cached
 * device address does not survive cudaDeviceReset: calls after a reset of
 * the device are not supported.  No reference counterpart. */
int gs_isect_sort_noalloc_check(int64_t n_isects, gs_stream_t stream);

/* Diagnostic of the bounded look-back wait, no reference counterpart: runs
 * the second 4096-key tile of one radix pass over n_isects keys (4096 <
 * n_isects <= 8192) alone, so that its wait on the first tile, which never
 * publishes, gives up after spin_limit polls (1..1024).  The pass then
 * raises the error word in `workspace` (gs_isect_sort_workspace_size bytes)
 * and finishes; gs_isect_sort_check reports GS_ERR_DEVICE.  The outputs get
 * the second tile's keys at in-range places, the rest is left untouched.
 * Lets a test run the give-up path without holding the GPU. */
int gs_isect_sort_wait_selftest(int64_t n_isects, const int64_t* isect_ids,
                                const int32_t* flatten_ids, int64_t* sorted_isect_ids,
                                int32_t* sorted_flatten_ids, void* workspace,
                                size_t workspace_bytes, uint32_t spin_limit,
                                gs_stream_t stream);

/* tile_offsets [I, tile_height, tile_width] int32 from sorted isect_ids:
 * lower bound of (image << tile_bits | tile) in isect_ids >> 32. */
int gs_isect_offset(int64_t n_isects, const int64_t* isect_ids, int32_t I,
                    int32_t tile_width, int32_t tile_height,
                    int32_t* tile_offsets, gs_stream_t stream);
/* The offsets of tile rows [tile_y0, tile_y1) only, into tile_offsets
 * [I, tile_y1 - tile_y0, tile_width] (a band of the image, with isect_ids
 * from an intersect call with the same window).  No reference counterpart. */
int gs_isect_offset_rows(int64_t n_isects, const int64_t* isect_ids, int32_t I,
                         int32_t tile_width, int32_t tile_height, int32_t tile_y0,
                         int32_t tile_y1, int32_t* tile_offsets, gs_stream_t stream);

/* Helper of the staged pipeline: tile_bits = floor(log2(n)) + 1, the
 * reference's floor_log2_plus_one (gsplat_intersect.cpp:60-65). */
int32_t gs_floor_log2_plus_one(int32_t value);

/* ------------------------------------------------------------------ */
/* rasterize to pixels (3DGS)                                          */
/* Replaces GSPlatRasterizeToPixels3DGS{,Backward}::eval_gpu,          */
/* gsplat_rasterize.cpp:572-724; params mirror                         */
/* RasterizeToPixels3DGSKernelParams, :28-40.                          */
/* ------------------------------------------------------------------ */
typedef struct {
  int32_t I, N, channels;
  int32_t image_width, image_height;
  int32_t tile_size, tile_width, tile_height;
  int64_t n_isects;
  int32_t use_backgrounds, use_masks;
  int32_t absgrad; /* bwd: write v_means2d_abs */
  int32_t tile_y0, tile_y1; /* when tile_y1 > tile_y0: only tile rows
                               [tile_y0, tile_y1) are rendered (a band;
                               tile_offsets is then [I, rows, tile_width] and
                               flatten_ids / n_isects the band's); else all */
  int32_t accumulate; /* bwd: add into the gradient outputs instead of
                         zeroing them first (bands after the first) */
  int32_t shared_opacities; /* when set, opacities and v_opacities are [N],
                               shared by the I images (entry g of the
                               flattened [I, N] index reads g mod N): the
                               per-Gaussian opacity of a multi-camera batch
                               without an [I, N] copy, and its gradient
                               summed over the images in place.  No
                               reference counterpart (the reference takes
                               [I, N]). */
  const float* sigma_bounds; /* optional, 8-byte aligned: the (keep, clamp)
                                sigma bounds of every opacity entry, laid out
                                like opacities ([I, N] or [N]) with two floats
                                each, from gs_rasterize_sigma_bounds.  Null:
                                the kernels derive them per staged entry
                                (same results, slower).  No reference
                                counterpart. */
  int32_t* tile_order;       /* optional scratch [slots = I * rows *
                                tile_width]: when given, each rasterizer call
                                first writes into it the order in which its
                                kernel takes the tiles -- costliest first
                                (gs_raster_tile_order: the forward by list
                                length, the backward by tile_cost when given)
                                -- so that no long tile is left to run alone
                                at the end of the grid.  Grids of more than
                                32768 tiles keep slot order (the scratch is
                                then left untouched).  The outputs do not
                                depend on it.  No reference counterpart. */
  int32_t* tile_cost;        /* optional [slots]: gs_rasterize_fwd writes per
                                tile the number of its list entries that its
                                pixels walk, max over the pixels of
                                (min(end - 1, last id) - start + 1) -- the
                                backward pass's work on the tile;
                                gs_rasterize_bwd orders its tiles by it.  No
                                reference counterpart. */
} gs_raster_params;

/* The tiles of p's grid (its band, when tile_y1 > tile_y0) in descending
 * order of their cost, at 1/8-octave resolution (bucket = 8 floor(log2 c) +
 * the next three bits of c), into tile_order [I * rows * tile_width]: what
 * the rasterizer calls write into p->tile_order before their kernels.  The
 * cost is tile_cost [slots] when given, else the intersection-list length
 * (p->n_isects and tile_offsets as for the rasterizer calls).  No reference
 * counterpart. */
int gs_raster_tile_order(const gs_raster_params* p, const int32_t* tile_offsets,
                         const int32_t* tile_cost, int32_t* tile_order,
                         gs_stream_t stream);

/* The exact alpha decisions of the rasterizer as two sigma bounds per
 * opacity: bounds[2i] = the largest sigma at which o = opacities[i] still
 * reaches alpha >= 1/255, bounds[2i+1] = the smallest sigma at which
 * o e^-sigma <= 0.99 (alpha not clamped), both with the correctly rounded
 * exponential and the reference's float multiply (-inf: never composited /
 * never clamped; NaN or +inf opacity: +inf, +inf; a -inf opacity, which the
 * reference composites at alpha 0.99 exactly where e^-sigma underflows to 0
 * (-inf * 0 is NaN, min(0.99, NaN) is 0.99): -103.972084, +inf, a negative
 * keep bound marking the range [103.972084, +inf]).  Pass them through
 * gs_raster_params.sigma_bounds.  With radii ([cameras, n, 2], 8-byte
 * aligned) only the entries some camera sees (both radii > 0) are written:
 * the others have no intersections, so no rasterizer reads them.  No
 * reference counterpart. */
int gs_rasterize_sigma_bounds(int64_t n, const float* opacities, const int32_t* radii,
                              int32_t cameras, float* bounds, gs_stream_t stream);

/* render_colors [I,H,W,ch], render_alphas [I,H,W,1], last_ids [I,H,W] */
int gs_rasterize_fwd(const gs_raster_params* p, const float* means2d,
                     const float* conics, const float* colors,
                     const float* opacities, const float* backgrounds,
                     const uint8_t* masks, const int32_t* tile_offsets,
                     const int32_t* flatten_ids, float* render_colors,
                     float* render_alphas, int32_t* last_ids,
                     gs_stream_t stream);
/* Gradient outputs are zeroed on the stream, then accumulated. */
int gs_rasterize_bwd(const gs_raster_params* p, const float* means2d,
                     const float* conics, const float* colors,
                     const float* opacities, const float* backgrounds,
                     const uint8_t* masks, const int32_t* tile_offsets,
                     const int32_t* flatten_ids, const float* render_alphas,
                     const int32_t* last_ids, const float* v_render_colors,
                     const float* v_render_alphas, float* v_means2d_abs,
                     float* v_means2d, float* v_conics, float* v_colors,
                     float* v_opacities, float* v_backgrounds,
                     gs_stream_t stream);

/* ------------------------------------------------------------------ */
/* training glue of the image-fitting trainer, on device               */
/* Replaces the MLX elementwise ops and mlx.optimizers.Adam of         */
/* scripts/test/train_image_fitting_3dgs_mlx.py (activations :33-36,   */
/* :104-118; Adam updates :529-566).  No kernel counterpart in the     */
/* reference (MLX runs these as generic array ops).                    */
/* ------------------------------------------------------------------ */

/* quats_n = quats / max(|quats|, 1e-8) [n,4] (16-byte aligned),
 * scales = exp(log_scales) [n,3], colors = sigmoid(color_logits) [n,3],
 * opacities = sigmoid(opacity_logits) [n]. */
int gs_fit_activate(int64_t n, const float* quats, const float* log_scales,
                    const float* color_logits, const float* opacity_logits,
                    float* quats_n, float* scales, float* colors, float* opacities,
                    gs_stream_t stream);

/* L2 image loss: v_render = 2 (render - target) / count and
 * *loss = mean((render - target)^2) (a device float; atomically summed, so
 * its last bits depend on the order of the CTAs). */
int gs_l2_loss_grad(int64_t count, const float* render, const float* target,
                    float* v_render, float* loss, gs_stream_t stream);

typedef struct {
  int64_t n;
  float learning_rate, beta1, beta2, eps; /* MLX Adam: 1e-2 (the trainer's
                                             lr), 0.9, 0.999, 1e-8 */
} gs_adam_params;

/* One Adam step (MLX semantics: no bias correction) on the raw parameters,
 * given the gradients of the activated ones (v_quats is d/d quats_n):
 * reverse mode of the activations, the update, the trainer's quaternion
 * renormalisation, and the activated parameters for the next step (written
 * into quats_n / scales / colors / opacities, which must hold this step's
 * activations on entry).  moment1 / moment2 [n,14] per Gaussian:
 * [means 3 | quats 4 | log_scales 3 | color_logits 3 | opacity 1]. */
int gs_fit_adam(const gs_adam_params* p, float* means, float* quats, float* log_scales,
                float* color_logits, float* opacity_logits, const float* v_means,
                const float* v_quats, const float* v_scales, const float* v_colors,
                const float* v_opacities, float* moment1, float* moment2,
                float* quats_n, float* scales, float* colors, float* opacities,
                gs_stream_t stream);

/* ------------------------------------------------------------------ */
/* Densification statistics of the reference trainer's default        */
/* strategy (scripts/test/scanner_points_training_utils.py,           */
/* ScannerDefaultStrategyRuntime) on device.                           */
/* ------------------------------------------------------------------ */
typedef struct {
  int32_t C, N;             /* cameras, Gaussians                       */
  int32_t width, height;    /* image size                               */
  int32_t n_cameras;        /* the gradient scale's camera factor       */
} gs_densify_params;

/* update_state (:412-451): for each (camera, Gaussian) with both radii
 * positive, grad2d[n] += |v_means2d[c,n] * (W/2, H/2) * n_cameras| and
 * count[n] += 1, cameras in order, fp32 as the reference (bit for bit).
 * With max_radii (the reference keeps it when refine_scale2d_stop_iter >
 * 0): max_radii[n] = max(max_radii[n], larger radius of the last camera
 * that sees n / max(W, H)).  v_means2d [C,N,2] (or the absgrad buffer),
 * radii [C,N,2]; grad2d, count, max_radii [N] are accumulated in place. */
int gs_densify_accumulate(const gs_densify_params* p, const float* v_means2d,
                          const int32_t* radii, float* grad2d, float* count,
                          float* max_radii, gs_stream_t stream);

typedef struct {
  int64_t n;                        /* Gaussians now                         */
  int64_t n_original;               /* split only below this index           */
  int32_t step;
  int32_t compute_grow;             /* clone and split masks                 */
  int32_t compute_prune;            /* prune mask                            */
  int32_t refine_scale2d_stop_iter; /* > 0: max_radii terms while step < it  */
  int32_t reset_every;              /* scale prunes only when step > it      */
  int32_t pad_;
  double grow_grad2d, grow_scale3d, grow_scale2d;
  double prune_opa, prune_scale3d, prune_scale2d, scene_scale;
} gs_densify_mask_params;

/* The refine masks (uint8, one per Gaussian): clone (:556-569), split
 * (:639-657) and prune (:706-718) -- the reference computes clone and split
 * from the same statistics (split skips the clones it appends) and prune
 * after both, so the caller asks for grow and prune in two calls around
 * its clone/split.  totals_device (int64[6]): clone, split, prune, prune by
 * opacity, by 3D scale, by 2D radius.  Decisions that need exp() can differ
 * from numpy's only within a few ulp of their thresholds. */
int gs_densify_masks(const gs_densify_mask_params* p, const float* grad2d,
                     const float* count, const float* max_radii,
                     const float* log_scales, const float* opacity_logits,
                     uint8_t* clone, uint8_t* split, uint8_t* prune,
                     int64_t* totals_device, gs_stream_t stream);

/* ------------------------------------------------------------------ */
/* SPZ export attributes                                               */
/* Replaces the numpy conversions of export_trained_spz               */
/* (scripts/test/scanner_points_training_utils.py:1424-1493, with     */
/* positions_to_spz :1361, scales_to_spz :1380, quats_to_spz :1392,   */
/* quats_to_spz_storage :1415): the arrays the reference hands to the */
/* spz package's GaussianCloud.  Packing them into a .spz file is that */
/* package's job (spz.save_spz), not this library's.                  */
/* ------------------------------------------------------------------ */
typedef struct {
  int64_t n;             /* Gaussians                                      */
  int32_t scale_mode;    /* 0 direct, 1 scanner_axis (y and z swapped)     */
  int32_t rotation_mode; /* 0 direct, 1 position_axis, 2 fastgs_conjugate,
                            3 position_conjugate                           */
  int32_t quat_order;    /* 0 wxyz, 1 xyzw                                 */
  int32_t color_mode;    /* 0 sh, 1 raw_rgb                                */
  int32_t source;        /* 0 SH model (colors_or_dc = features_dc [n,3]),
                            1 RGB model (colors_or_dc = its colours [n,3]) */
  int32_t sh_rest;       /* rest coefficients written per Gaussian:
                            (degree+1)^2 - 1 for an SH model in sh mode,
                            else 0                                         */
  int32_t rest_stride;   /* rest coefficients per row of features_rest     */
} gs_spz_params;

/* means [n,3], quats [n,4] (wxyz), log_scales [n,3], opacity_logits [n],
 * colors_or_dc [n,3], features_rest [n,rest_stride,3] -> positions [n,3],
 * scales [n,3], rotations [n,4], alphas [n], colors [n,3],
 * sh [n,sh_rest,3] (NULL when sh_rest is 0).  fp32 in the reference's
 * operation order. */
int gs_spz_attributes(const gs_spz_params* p, const float* means,
                      const float* quats, const float* log_scales,
                      const float* opacity_logits, const float* colors_or_dc,
                      const float* features_rest, float* positions,
                      float* scales, float* rotations, float* alphas,
                      float* colors, float* sh, gs_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* GSPLAT_B200_H */
