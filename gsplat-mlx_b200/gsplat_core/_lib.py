"""ctypes binding of libgsplat_b200.so (the C ABI declared in
include/gsplat_b200.h).

The shared library is the product's compute path; there is no fallback.
Loading fails loudly when the library is missing or when no CUDA device is
usable for a call.
"""
from __future__ import annotations

import ctypes as ct
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("GSPLAT_B200_LIB", os.path.join(_HERE, "libgsplat_b200.so"))

_vp = ct.c_void_p
_i32 = ct.c_int32
_i64 = ct.c_int64
_f = ct.c_float
_sz = ct.c_size_t

GS_OK = 0
GS_ERR_INVALID = 1
GS_ERR_UNSUPPORTED = 2
GS_ERR_OVERFLOW = 3
GS_ERR_CUDA = 4
GS_ERR_WORKSPACE = 5


class QS2CParams(ct.Structure):
    _fields_ = [("n", _i64), ("compute_covar", _i32), ("compute_preci", _i32), ("triu", _i32)]


class ProjectionParams(ct.Structure):
    _fields_ = [("B", _i32), ("C", _i32), ("N", _i32), ("image_width", _i32),
                ("image_height", _i32), ("eps2d", _f), ("near_plane", _f), ("far_plane", _f),
                ("radius_clip", _f), ("calc_compensations", _i32), ("camera_model", _i32),
                ("use_covars", _i32), ("use_opacities", _i32)]


class SHParams(ct.Structure):
    _fields_ = [("n", _i64), ("K", _i32), ("degrees_to_use", _i32), ("use_masks", _i32)]


class SHGlueParams(ct.Structure):
    _fields_ = [("C", _i32), ("N", _i32), ("K", _i32), ("degrees_to_use", _i32),
                ("use_masks", _i32), ("skip_zero_cotangents", _i32), ("camera_groups", _i32)]


class DensifyParams(ct.Structure):
    _fields_ = [("C", _i32), ("N", _i32), ("width", _i32), ("height", _i32), ("n_cameras", _i32)]


class DensifyMaskParams(ct.Structure):
    _fields_ = [("n", _i64), ("n_original", _i64), ("step", _i32), ("compute_grow", _i32),
                ("compute_prune", _i32), ("refine_scale2d_stop_iter", _i32),
                ("reset_every", _i32), ("pad_", _i32), ("grow_grad2d", ct.c_double),
                ("grow_scale3d", ct.c_double), ("grow_scale2d", ct.c_double),
                ("prune_opa", ct.c_double), ("prune_scale3d", ct.c_double),
                ("prune_scale2d", ct.c_double), ("scene_scale", ct.c_double)]


class SpzParams(ct.Structure):
    _fields_ = [("n", _i64), ("scale_mode", _i32), ("rotation_mode", _i32), ("quat_order", _i32),
                ("color_mode", _i32), ("source", _i32), ("sh_rest", _i32), ("rest_stride", _i32)]


class AdamParams(ct.Structure):
    _fields_ = [("n", _i64), ("learning_rate", _f), ("beta1", _f), ("beta2", _f), ("eps", _f)]


class IsectParams(ct.Structure):
    _fields_ = [("I", _i32), ("N", _i32), ("tile_size", _i32), ("tile_width", _i32),
                ("tile_height", _i32), ("tile_y0", _i32), ("tile_y1", _i32),
                ("reuse_depth_order", _i32), ("positive_depths", _i32),
                ("shared_opacities", _i32)]


class RasterParams(ct.Structure):
    _fields_ = [("I", _i32), ("N", _i32), ("channels", _i32), ("image_width", _i32),
                ("image_height", _i32), ("tile_size", _i32), ("tile_width", _i32),
                ("tile_height", _i32), ("n_isects", _i64), ("use_backgrounds", _i32),
                ("use_masks", _i32), ("absgrad", _i32), ("tile_y0", _i32), ("tile_y1", _i32),
                ("accumulate", _i32), ("shared_opacities", _i32), ("sigma_bounds", _vp),
                ("tile_order", _vp), ("tile_cost", _vp)]


_P = ct.POINTER

# (name, restype, argtypes); every exported symbol of include/gsplat_b200.h.
SIGNATURES = {
    "gs_status_string": (ct.c_char_p, [ct.c_int]),
    "gs_last_error": (ct.c_char_p, []),
    "gs_version": (ct.c_int, []),
    "gs_floor_log2_plus_one": (_i32, [_i32]),
    "gs_quat_scale_to_covar_fwd": (ct.c_int, [_P(QS2CParams), _vp, _vp, _vp, _vp, _vp]),
    "gs_quat_scale_to_covar_bwd": (ct.c_int, [_P(QS2CParams), _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "gs_projection_fwd": (ct.c_int, [_P(ProjectionParams)] + [_vp] * 13),
    "gs_projection_bwd": (ct.c_int, [_P(ProjectionParams)] + [_vp] * 19),
    "gs_sh_fwd": (ct.c_int, [_P(SHParams), _vp, _vp, _vp, _vp, _vp]),
    "gs_sh_bwd": (ct.c_int, [_P(SHParams), _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "gs_sh_glue_fwd": (ct.c_int, [_P(SHGlueParams), _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "gs_sh_glue_bwd": (ct.c_int, [_P(SHGlueParams), _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "gs_isect_tile_count": (ct.c_int, [_P(IsectParams), _vp, _vp, _vp, _vp]),
    "gs_isect_tile_count_total": (ct.c_int, [_P(IsectParams), _vp, _vp, _vp, _vp, _vp]),
    "gs_isect_scan_workspace_size": (_sz, [_i64]),
    "gs_isect_scan": (ct.c_int, [_i64, _vp, _vp, _vp, _vp, _sz, _vp]),
    "gs_isect_tile_encode": (ct.c_int, [_P(IsectParams), _vp, _vp, _vp, _vp, _i64, _vp, _vp, _vp]),
    "gs_isect_tile_encode_sorted_workspace_size": (_sz, [_i64, _i64]),
    "gs_isect_tile_encode_sorted": (ct.c_int, [_P(IsectParams), _vp, _vp, _vp, _vp, _i64, _vp, _vp,
                                               _vp, _sz, _vp]),
    "gs_isect_tile_encode_sorted_check": (ct.c_int, [_i64, _i64, _vp, _vp]),
    "gs_isect_tile_count_totals": (ct.c_int, [_P(IsectParams), _vp, _vp, _vp, _vp, _vp]),
    "gs_isect_tile_encode_binned_workspace_size": (_sz, [_P(IsectParams), _i64]),
    "gs_isect_tile_encode_binned": (ct.c_int, [_P(IsectParams), _vp, _vp, _vp, _i64, _i64, _vp,
                                               _vp, _vp, _vp, _sz, _vp]),
    "gs_isect_tile_encode_binned_culled": (ct.c_int, [_P(IsectParams), _vp, _vp, _vp, _vp, _vp,
                                                      _i64, _i64, _vp, _vp, _vp, _vp, _vp, _sz,
                                                      _vp]),
    "gs_isect_tile_encode_binned_check": (ct.c_int, [_i64, _vp, _vp]),
    "gs_store_to_host_i64": (ct.c_int, [_vp, _vp, _i32, _vp]),
    "gs_pack_visible_workspace_size": (_sz, [_i64]),
    "gs_pack_visible": (ct.c_int, [_i64, _i32] + [_vp] * 5 + [_i64] + [_vp] * 9 + [_sz, _vp]),
    "gs_isect_tile_encode_binned_packed_workspace_size": (_sz, [_P(IsectParams), _i64]),
    "gs_isect_tile_encode_binned_packed": (ct.c_int, [_P(IsectParams), _vp, _vp, _vp, _vp, _i64,
                                                      _i64, _vp, _vp, _vp, _vp, _sz, _vp]),
    "gs_isect_sort_check": (ct.c_int, [_i64, _vp, _vp]),
    "gs_isect_sort_workspace_size": (_sz, [_i64]),
    "gs_isect_sort": (ct.c_int, [_i64, _i32, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "gs_isect_offset": (ct.c_int, [_i64, _vp, _i32, _i32, _i32, _vp, _vp]),
    "gs_isect_offset_rows": (ct.c_int, [_i64, _vp, _i32, _i32, _i32, _i32, _i32, _vp, _vp]),
    "gs_isect_sort_noalloc": (ct.c_int, [_i64, _i32, _vp, _vp, _vp, _vp, _vp]),
    "gs_isect_sort_noalloc_check": (ct.c_int, [_i64, _vp]),
    "gs_rasterize_sigma_bounds": (ct.c_int, [_i64, _vp, _vp, _i32, _vp, _vp]),
    "gs_raster_tile_order": (ct.c_int, [_vp, _vp, _vp, _vp, _vp]),
    "gs_isect_sort_wait_selftest": (ct.c_int, [_i64, _vp, _vp, _vp, _vp, _vp, _sz,
                                               ct.c_uint32, _vp]),
    "gs_fit_activate": (ct.c_int, [_i64] + [_vp] * 9),
    "gs_l2_loss_grad": (ct.c_int, [_i64] + [_vp] * 5),
    "gs_fit_adam": (ct.c_int, [_P(AdamParams)] + [_vp] * 17),
    "gs_densify_accumulate": (ct.c_int, [_P(DensifyParams)] + [_vp] * 6),
    "gs_densify_masks": (ct.c_int, [_P(DensifyMaskParams)] + [_vp] * 10),
    "gs_spz_attributes": (ct.c_int, [_P(SpzParams)] + [_vp] * 13),
    "gs_rasterize_fwd": (ct.c_int, [_P(RasterParams)] + [_vp] * 12),
    "gs_rasterize_bwd": (ct.c_int, [_P(RasterParams)] + [_vp] * 19),
}

_lib = None


def load(path: str = LIB_PATH) -> ct.CDLL:
    """Load the native library once and declare every entry point."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise RuntimeError(
            f"gsplat_b200 native library not found at {path}; build it with "
            f"`python gsplat-mlx_b200/build.py` (there is no CPU fallback)")
    lib = ct.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


class GsplatError(RuntimeError):
    """Error status returned by the native library."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


def check(status: int, what: str) -> None:
    if status != GS_OK:
        lib = load()
        msg = lib.gs_last_error().decode(errors="replace")
        kind = lib.gs_status_string(status).decode()
        raise GsplatError(status, f"{what}: {msg} [{kind}]" if msg else f"{what} [{kind}]")
