"""Drop-in mirror of the reference's ``_gsplat_core`` module
(gsplat_core/binding/binding.cpp:447-534): the same ten operator functions
(plus the two template dummies) with the same names, keyword arguments,
defaults, dict keys, output shapes / dtypes and error messages.

Arrays are CUDA ``torch.Tensor`` s (numpy arrays are accepted and moved to
the current device).  Every operator runs the sm_100a kernels of
``libgsplat_b200.so`` through its C ABI on the current torch CUDA stream;
torch only provides device memory and the stream.  Missing optional keys
behave like the reference's empty ``zeros({0})`` arrays
(binding.cpp:37-45); missing required keys raise ``RuntimeError``
(binding.cpp:26-35).  Outputs are zero-filled where the reference leaves
zeros (culled / masked entries), and optional outputs that are not
requested have shape ``[0]``.
"""
from __future__ import annotations

import ctypes as ct
import math

import numpy as np
import torch

from . import _lib
from ._lib import (IsectParams, ProjectionParams, QS2CParams, RasterParams, SHGlueParams,
                   SHParams, check)

__all__ = [
    "dummy_add", "dummy_array_add",
    "projection_ewa_3dgs_fused_forward", "projection_ewa_3dgs_fused_backward",
    "intersect_tile_forward", "intersect_offset_forward",
    "rasterize_to_pixels_3dgs_forward", "rasterize_to_pixels_3dgs_backward",
    "spherical_harmonics_forward", "spherical_harmonics_backward",
    "quat_scale_to_covar_preci_forward", "quat_scale_to_covar_preci_backward",
]

# ---------------------------------------------------------------- plumbing


def _device():
    if not torch.cuda.is_available():
        raise RuntimeError("gsplat_core: no CUDA device (there is no CPU fallback)")
    return torch.device("cuda", torch.cuda.current_device())


def _stream():
    return ct.c_void_p(torch.cuda.current_stream().cuda_stream)


def _arr(x):
    """Tensor view of an input (numpy arrays are wrapped, not copied).
    Shapes are validated on whatever device the array lives on; _cuda()
    moves validated host arrays to the device."""
    if x is None:
        return None
    if isinstance(x, np.ndarray):
        x = torch.from_numpy(np.ascontiguousarray(x))
    if not isinstance(x, torch.Tensor):
        x = torch.as_tensor(x)
    return x


def _cuda(*ts):
    """Contiguous device copies (mx::contiguous) of validated inputs."""
    dev = _device()
    out = []
    for t in ts:
        if t is not None:
            if t.device.type != "cuda":
                t = t.to(dev)
            t = t.contiguous()
        out.append(t)
    return out if len(out) != 1 else out[0]


def _opt(inputs, key):
    """get_or_empty (binding.cpp:37-45): absent or empty -> None."""
    v = inputs.get(key) if inputs is not None else None
    if v is None:
        return None
    v = _arr(v)
    return v if v.numel() != 0 else None


def _req(inputs, key):
    """require_key (binding.cpp:26-35)."""
    if inputs is None or key not in inputs or inputs[key] is None:
        raise RuntimeError(f"gsplat_core binding missing input: {key}")
    return _arr(inputs[key])


def _ptr(t):
    return None if t is None else ct.c_void_p(t.data_ptr())


def _empty(shape, dtype=torch.float32):
    return torch.empty(shape, dtype=dtype, device=_device())


def _zeros0(dtype=torch.float32):
    return torch.zeros((0,), dtype=dtype, device=_device())


def _as_bool_u8(m):
    if m is None:
        return None
    if m.dtype not in (torch.bool, torch.uint8):
        m = m != 0
    return m


# ---------------------------------------------------------------- dummies


def dummy_add(a: int, b: int) -> int:
    """Template leftover of the reference (gsplat_core/dummy.cpp)."""
    return a + b


def dummy_array_add(inputs):
    """Template leftover of the reference (binding.cpp:57-61)."""
    return _req(inputs, "a") + _req(inputs, "b")


# ---------------------------------------------------------------- projection


def _projection_shapes(means, viewmats, Ks):
    """gsplat_projection.cpp:67-141 shape rules."""
    if means.dim() < 2 or means.shape[-1] != 3:
        raise RuntimeError("means must have shape [..., N, 3].")
    if viewmats.dim() < 3 or viewmats.shape[-1] != 4 or viewmats.shape[-2] != 4:
        raise RuntimeError("viewmats must have shape [..., C, 4, 4].")
    if Ks.dim() < 3 or Ks.shape[-1] != 3 or Ks.shape[-2] != 3:
        raise RuntimeError("Ks must have shape [..., C, 3, 3].")
    N = means.shape[-2]
    C = viewmats.shape[-3]
    B = means.numel() // (N * 3) if N > 0 else int(np.prod(means.shape[:-2]))
    if viewmats.numel() != B * C * 16 or Ks.numel() != B * C * 9:
        raise RuntimeError("viewmats and Ks must have shape [B, C, 4, 4] and [B, C, 3, 3].")
    prefix = tuple(means.shape[:-2]) + (C, N)
    return B, C, N, prefix


def projection_ewa_3dgs_fused_forward(inputs, image_width, image_height, eps2d=0.3,
                                      near_plane=0.01, far_plane=1.0e10, radius_clip=0.0,
                                      calc_compensations=False, camera_model=0):
    """binding.cpp:63-117 / gsplat_projection.cpp:584-618 (GPU semantics of
    metal/gsplat_projection.metal:214-339)."""
    means = _req(inputs, "means")
    viewmats = _req(inputs, "viewmats")
    Ks = _req(inputs, "Ks")
    covars = _opt(inputs, "covars")
    quats = _opt(inputs, "quats")
    scales = _opt(inputs, "scales")
    opacities = _opt(inputs, "opacities")
    vsp_in = inputs.get("viewspace_points") if inputs is not None else None
    viewspace_points = _arr(vsp_in) if vsp_in is not None else torch.zeros((0,))
    use_covars = covars is not None
    use_opacities = opacities is not None
    B, C, N, prefix = _projection_shapes(means, viewmats, Ks)
    if not use_covars and (quats is None or scales is None):
        raise RuntimeError("projection_ewa_3dgs_fused_forward expects covars or quats+scales.")
    if viewspace_points.numel() != 0 and tuple(viewspace_points.shape) != prefix + (2,):
        raise RuntimeError("viewspace_points must have shape [..., C, N, 2].")
    if use_covars and covars.numel() != B * N * 6:
        raise RuntimeError("covars must have shape [..., N, 6].")
    if not use_covars and (quats.numel() != B * N * 4 or scales.numel() != B * N * 3):
        raise RuntimeError("quats and scales must have shapes [..., N, 4] and [..., N, 3].")
    if use_opacities and opacities.numel() != B * N:
        raise RuntimeError("opacities must have shape [..., N].")
    for t in (means, viewmats, Ks, covars, quats, scales, opacities):
        if t is not None and t.dtype != torch.float32:
            raise RuntimeError("projection_ewa_3dgs_fused_forward expects float32 inputs.")
    means, viewmats, Ks, covars, quats, scales, opacities = _cuda(
        means, viewmats, Ks, covars, quats, scales, opacities)
    out = {
        "radii": _empty(prefix + (2,), torch.int32),
        "means2d": _empty(prefix + (2,)),
        "depths": _empty(prefix),
        "conics": _empty(prefix + (3,)),
        "compensations": _empty(prefix) if calc_compensations else _zeros0(),
    }
    p = ProjectionParams(B, C, N, int(image_width), int(image_height), float(eps2d),
                         float(near_plane), float(far_plane), float(radius_clip),
                         int(bool(calc_compensations)), int(camera_model), int(use_covars),
                         int(use_opacities))
    lib = _lib.load()
    check(lib.gs_projection_fwd(ct.byref(p), _ptr(means), _ptr(covars), _ptr(quats),
                                _ptr(scales), _ptr(opacities), _ptr(viewmats), _ptr(Ks),
                                _ptr(out["means2d"]), _ptr(out["depths"]), _ptr(out["conics"]),
                                _ptr(out["compensations"]) if calc_compensations else None,
                                _ptr(out["radii"]), _stream()),
          "projection_ewa_3dgs_fused_forward")
    # Passed through unchanged; it only carries the means2d cotangent in
    # the autograd wiring (gsplat_projection.cpp:1200-1201).
    out["viewspace_points"] = viewspace_points if viewspace_points.numel() else _zeros0()
    return out


def projection_ewa_3dgs_fused_backward(inputs, forward_outputs, cotangents, image_width,
                                       image_height, eps2d=0.3, camera_model=0,
                                       viewmats_requires_grad=False):
    """binding.cpp:119-186 / gsplat_projection.cpp:620-652 (eval_gpu math
    of metal/gsplat_projection.metal:446-676)."""
    means = _req(inputs, "means")
    viewmats = _req(inputs, "viewmats")
    Ks = _req(inputs, "Ks")
    covars = _opt(inputs, "covars")
    quats = _opt(inputs, "quats")
    scales = _opt(inputs, "scales")
    radii = _req(forward_outputs, "radii")
    conics = _req(forward_outputs, "conics")
    compensations = _opt(forward_outputs, "compensations")
    v_means2d = _req(cotangents, "v_means2d")
    v_depths = _req(cotangents, "v_depths")
    v_conics = _req(cotangents, "v_conics")
    v_compensations = _opt(cotangents, "v_compensations")
    use_covars = covars is not None
    B, C, N, prefix = _projection_shapes(means, viewmats, Ks)
    if not use_covars and (quats is None or scales is None):
        raise RuntimeError("projection_ewa_3dgs_fused_forward expects covars or quats+scales.")
    if int(camera_model) != 0:
        raise RuntimeError("projection_ewa_3dgs_fused_backward currently supports pinhole only.")
    if radii.dtype != torch.int32:
        raise RuntimeError("radii must be int32.")
    if (tuple(v_means2d.shape) != prefix + (2,) or tuple(v_conics.shape) != prefix + (3,)
            or tuple(v_depths.shape) != prefix):
        raise RuntimeError("projection backward cotangent shape mismatch.")
    if radii.numel() != B * C * N * 2 or conics.numel() != B * C * N * 3:
        raise RuntimeError("projection backward forward-output shape mismatch.")
    calc_comp = compensations is not None
    if calc_comp and v_compensations is not None and v_compensations.numel() != B * C * N:
        raise RuntimeError("projection backward cotangent shape mismatch.")
    (means, viewmats, Ks, covars, quats, scales, radii, conics, compensations, v_means2d,
     v_depths, v_conics, v_compensations) = _cuda(
        means, viewmats, Ks, covars, quats, scales, radii, conics, compensations, v_means2d,
        v_depths, v_conics, v_compensations)
    out = {"v_means": _empty(tuple(means.shape))}
    if use_covars:
        out["v_covars"] = _empty(tuple(covars.shape))
    else:
        out["v_quats"] = _empty(tuple(quats.shape))
        out["v_scales"] = _empty(tuple(scales.shape))
    if viewmats_requires_grad:
        out["v_viewmats"] = _empty(tuple(viewmats.shape))
    p = ProjectionParams(B, C, N, int(image_width), int(image_height), float(eps2d), -1.0e20,
                         1.0e20, 0.0, int(calc_comp), 0, int(use_covars), 0)
    lib = _lib.load()
    check(lib.gs_projection_bwd(ct.byref(p), _ptr(means), _ptr(covars), _ptr(quats),
                                _ptr(scales), _ptr(viewmats), _ptr(Ks), _ptr(radii),
                                _ptr(conics), _ptr(compensations), _ptr(v_means2d),
                                _ptr(v_depths), _ptr(v_conics),
                                _ptr(v_compensations) if calc_comp else None,
                                _ptr(out["v_means"]), _ptr(out.get("v_covars")),
                                _ptr(out.get("v_quats")), _ptr(out.get("v_scales")),
                                _ptr(out.get("v_viewmats")), _stream()),
          "projection_ewa_3dgs_fused_backward")
    return out


# ---------------------------------------------------------------- intersect


def floor_log2_plus_one(value: int) -> int:
    """gsplat_intersect.cpp:60-65 (float log2, as the reference)."""
    if value <= 0:
        raise RuntimeError("intersect expects positive image/tile counts.")
    return int(_lib.load().gs_floor_log2_plus_one(int(value)))


def _validate_intersect(means2d, radii, depths, conics, opacities, image_ids, gaussian_ids,
                        segmented):
    """gsplat_intersect.cpp:114-144."""
    if image_ids is not None or gaussian_ids is not None:
        raise RuntimeError("intersect_tile packed path is not implemented yet.")
    if segmented:
        raise RuntimeError("intersect_tile segmented sort is not implemented yet.")
    if conics is not None or opacities is not None:
        raise RuntimeError("intersect_tile AccuTile conics/opacities path is not implemented yet.")
    if means2d.dim() < 3 or means2d.shape[-1] != 2:
        raise RuntimeError("means2d must have shape [..., N, 2].")
    if radii.dim() != means2d.dim() or radii.shape[-1] != 2:
        raise RuntimeError("radii must have shape [..., N, 2].")
    if depths.dim() + 1 != means2d.dim():
        raise RuntimeError("depths must have shape [..., N].")
    if means2d.dtype != torch.float32 or radii.dtype != torch.int32 or depths.dtype != torch.float32:
        raise RuntimeError(
            "intersect_tile dense path expects float32 means2d/depths and int32 radii.")


def intersect_tile_count(means2d, radii, I, tile_size, tile_width, tile_height):
    """GSPlatIntersectTileCount (gsplat_intersect.cpp:174-194, 342-382)."""
    N = means2d.shape[-2]
    numel = radii.numel() // 2
    if I <= 0 or numel % I != 0 or numel != I * N:
        raise RuntimeError("intersect_tile_count dense path expects depths size to equal I * N.")
    out = _empty(tuple(radii.shape[:-1]), torch.int32)
    p = IsectParams(int(I), int(N), int(tile_size), int(tile_width), int(tile_height))
    check(_lib.load().gs_isect_tile_count(ct.byref(p), _ptr(means2d), _ptr(radii), _ptr(out),
                                          _stream()), "intersect_tile_count")
    return out


def intersect_tile_offsets(tiles_per_gauss):
    """Exclusive cumsum of the per-Gaussian counts (gsplat_intersect.cpp:
    196-211) and the host-read total (:155-170, the one sync per call)."""
    if tiles_per_gauss.dtype != torch.int32:
        raise RuntimeError("intersect_tile_offsets expects int32 tiles_per_gauss.")
    n = tiles_per_gauss.numel()
    offsets = _empty(tuple(tiles_per_gauss.shape), torch.int32)
    total = torch.zeros((1,), dtype=torch.int64, device=_device())
    lib = _lib.load()
    ws = _empty((max(1, lib.gs_isect_scan_workspace_size(n)),), torch.uint8)
    check(lib.gs_isect_scan(n, _ptr(tiles_per_gauss), _ptr(offsets), _ptr(total), _ptr(ws),
                            ws.numel(), _stream()), "intersect_tile_offsets")
    return offsets, total


def intersect_tile_encode(means2d, radii, depths, tile_offsets, I, tile_size, tile_width,
                          tile_height, total_isects):
    """GSPlatIntersectTileEncode (gsplat_intersect.cpp:213-264, 488-539)."""
    N = means2d.shape[-2]
    if total_isects < 0:
        raise RuntimeError("intersect_tile_encode expects non-negative total_isects.")
    if total_isects >= 2 ** 31:
        raise RuntimeError(
            f"intersect_tile_encode: {total_isects} intersections exceed the int32 index range")
    isect_ids = _empty((total_isects,), torch.int64)
    flatten_ids = _empty((total_isects,), torch.int32)
    p = IsectParams(int(I), int(N), int(tile_size), int(tile_width), int(tile_height))
    check(_lib.load().gs_isect_tile_encode(ct.byref(p), _ptr(means2d), _ptr(radii), _ptr(depths),
                                           _ptr(tile_offsets), int(total_isects), _ptr(isect_ids),
                                           _ptr(flatten_ids), _stream()),
          "intersect_tile_encode")
    return isect_ids, flatten_ids


def intersect_tile_encode_sorted(means2d, radii, depths, tiles_per_gauss, I, tile_size,
                                 tile_width, tile_height, total_isects):
    """Encode + stable sort in one native call (the sort=True branch of
    gsplat_intersect.cpp:288-307); bit-identical to encode then sort."""
    N = means2d.shape[-2]
    if total_isects < 0:
        raise RuntimeError("intersect_tile_encode expects non-negative total_isects.")
    if total_isects >= 2 ** 31:
        raise RuntimeError(
            f"intersect_tile_encode: {total_isects} intersections exceed the int32 index range")
    isect_ids = _empty((total_isects,), torch.int64)
    flatten_ids = _empty((total_isects,), torch.int32)
    if total_isects == 0:
        return isect_ids, flatten_ids
    lib = _lib.load()
    ws = _empty((lib.gs_isect_tile_encode_sorted_workspace_size(int(I) * int(N), total_isects),),
                torch.uint8)
    p = IsectParams(int(I), int(N), int(tile_size), int(tile_width), int(tile_height))
    check(lib.gs_isect_tile_encode_sorted(ct.byref(p), _ptr(means2d), _ptr(radii), _ptr(depths),
                                          _ptr(tiles_per_gauss), int(total_isects),
                                          _ptr(isect_ids), _ptr(flatten_ids), _ptr(ws), ws.numel(),
                                          _stream()), "intersect_tile_encode_sorted")
    return isect_ids, flatten_ids


def intersect_tile_count_totals(means2d, radii, I, tile_size, tile_width, tile_height):
    """Tile counts per (image, Gaussian) and, read on the host, the totals
    of intersections and of the binned encode's entries."""
    N = means2d.shape[-2]
    numel = radii.numel() // 2
    if I <= 0 or numel % I != 0 or numel != I * N:
        raise RuntimeError("intersect_tile_count dense path expects depths size to equal I * N.")
    out = _empty(tuple(radii.shape[:-1]), torch.int32)
    totals = torch.zeros((2,), dtype=torch.int64, device=_device())
    p = IsectParams(int(I), int(N), int(tile_size), int(tile_width), int(tile_height))
    check(_lib.load().gs_isect_tile_count_totals(ct.byref(p), _ptr(means2d), _ptr(radii),
                                                 _ptr(out), _ptr(totals), _stream()),
          "intersect_tile_count")
    m, bins = (int(v) for v in totals.tolist())
    return out, m, bins


def intersect_tile_encode_binned(means2d, radii, depths, I, tile_size, tile_width, tile_height,
                                 total_isects, n_bin_entries, tile_offsets=None):
    """Encode + stable sort through 4x4-tile bins (one native call);
    bit-identical to encode then sort.  With ``tile_offsets`` (int32
    [I, tile_height, tile_width]) the tile offsets are written too."""
    N = means2d.shape[-2]
    if total_isects < 0:
        raise RuntimeError("intersect_tile_encode expects non-negative total_isects.")
    if total_isects >= 2 ** 31:
        raise RuntimeError(
            f"intersect_tile_encode: {total_isects} intersections exceed the int32 index range")
    isect_ids = _empty((total_isects,), torch.int64)
    flatten_ids = _empty((total_isects,), torch.int32)
    lib = _lib.load()
    p = IsectParams(int(I), int(N), int(tile_size), int(tile_width), int(tile_height))
    ws = _empty((max(1, lib.gs_isect_tile_encode_binned_workspace_size(ct.byref(p),
                                                                      n_bin_entries)),),
                torch.uint8)
    check(lib.gs_isect_tile_encode_binned(ct.byref(p), _ptr(means2d), _ptr(radii), _ptr(depths),
                                          int(total_isects), int(n_bin_entries), _ptr(isect_ids),
                                          _ptr(flatten_ids), _ptr(tile_offsets), _ptr(ws),
                                          ws.numel(), _stream()), "intersect_tile_encode_binned")
    return isect_ids, flatten_ids


def intersect_tile_culled_forward(inputs, I, tile_size, tile_width, tile_height):
    """Sorted intersections with opacity-aware tile culling: what
    ``intersect_tile_forward(..., sort=True)`` returns, minus every
    (tile, Gaussian) pair whose Gaussian -- conics [I,N,3] and opacities
    [I,N], the rasterizer's inputs -- stays below alpha 1/255 at every pixel
    centre of the tile.  The reference's intersect_tile_forward refuses
    conics / opacities (gsplat_intersect.cpp:115-126); the rasterizer skips
    such pairs at every pixel, so rendering these lists gives the same
    colours and alphas bit for bit.  Returns {"isect_ids", "flatten_ids",
    "tile_offsets"} (the kept pairs, in the unculled order; tile_offsets
    [I, tile_height, tile_width] into them)."""
    means2d = _req(inputs, "means2d")
    radii = _req(inputs, "radii")
    depths = _req(inputs, "depths")
    conics = _req(inputs, "conics")
    opacities = _req(inputs, "opacities")
    _validate_intersect(means2d, radii, depths, None, None, None, None, False)
    means2d, radii, depths = _cuda(means2d, radii, depths)
    if conics.dtype != torch.float32 or opacities.dtype != torch.float32:
        raise RuntimeError("intersect_tile_culled_forward expects float32 conics / opacities.")
    conics, opacities = _cuda(conics, opacities)
    N = means2d.shape[-2]
    if conics.numel() != int(I) * N * 3 or opacities.numel() != int(I) * N:
        raise RuntimeError("intersect_tile_culled_forward expects conics [I,N,3] and "
                           "opacities [I,N].")
    if max(tile_width, tile_height) > 65535:
        raise RuntimeError("intersect_tile_culled_forward: more than 65535 tiles per row or column.")
    if floor_log2_plus_one(I) + floor_log2_plus_one(tile_width * tile_height) > 32:
        raise RuntimeError("intersect_tile_encode image id and tile id require more than 32 bits.")
    _, m, bins = intersect_tile_count_totals(means2d, radii, I, tile_size, tile_width, tile_height)
    if m >= 2 ** 31:
        raise RuntimeError(
            f"intersect_tile_encode: {m} intersections exceed the int32 index range")
    isect_ids = _empty((m,), torch.int64)
    flatten_ids = _empty((m,), torch.int32)
    offsets = _empty((int(I), int(tile_height), int(tile_width)), torch.int32)
    kept = torch.zeros((1,), dtype=torch.int64, device=means2d.device)
    lib = _lib.load()
    p = IsectParams(int(I), int(N), int(tile_size), int(tile_width), int(tile_height))
    ws = _empty((max(1, lib.gs_isect_tile_encode_binned_workspace_size(ct.byref(p), bins)),),
                torch.uint8)
    check(lib.gs_isect_tile_encode_binned_culled(
        ct.byref(p), _ptr(means2d), _ptr(radii), _ptr(depths), _ptr(conics),
        _ptr(opacities), int(m), int(bins), _ptr(isect_ids), _ptr(flatten_ids),
        _ptr(offsets), _ptr(kept), _ptr(ws), ws.numel(), _stream()),
        "intersect_tile_culled_forward")
    if bins > 0:
        check(lib.gs_isect_tile_encode_binned_check(bins, _ptr(ws), _stream()),
              "intersect_tile_culled_forward")
    gap = m - int(kept.item())  # the kept lists fill the last places
    return {"isect_ids": isect_ids[gap:], "flatten_ids": flatten_ids[gap:],
            "tile_offsets": offsets - gap}


def intersect_tile_sort(isect_ids, flatten_ids, key_bits=64):
    """Stable sort by key (gsplat_intersect.cpp:266-286: argsort + take)."""
    if isect_ids.dtype != torch.int64:
        raise RuntimeError("intersect_tile_sort expects int64 isect_ids.")
    if flatten_ids.dtype != torch.int32:
        raise RuntimeError("intersect_tile_sort expects int32 flatten_ids.")
    if isect_ids.dim() != 1 or flatten_ids.dim() != 1 or isect_ids.numel() != flatten_ids.numel():
        raise RuntimeError("intersect_tile_sort expects matching 1D isect_ids and flatten_ids.")
    m = isect_ids.numel()
    out_ids = _empty((m,), torch.int64)
    out_f = _empty((m,), torch.int32)
    if m == 0:
        return out_ids, out_f
    lib = _lib.load()
    ws = _empty((lib.gs_isect_sort_workspace_size(m),), torch.uint8)
    check(lib.gs_isect_sort(m, int(key_bits), _ptr(isect_ids), _ptr(flatten_ids), _ptr(out_ids),
                            _ptr(out_f), _ptr(ws), ws.numel(), _stream()), "intersect_tile_sort")
    return out_ids, out_f


def intersect_tile_forward(inputs, I, tile_size, tile_width, tile_height, sort=True,
                           segmented=False):
    """binding.cpp:188-232 / gsplat_intersect.cpp:288-307."""
    means2d = _req(inputs, "means2d")
    radii = _req(inputs, "radii")
    depths = _req(inputs, "depths")
    conics = _opt(inputs, "conics")
    opacities = _opt(inputs, "opacities")
    image_ids = _opt(inputs, "image_ids")
    gaussian_ids = _opt(inputs, "gaussian_ids")
    _validate_intersect(means2d, radii, depths, conics, opacities, image_ids, gaussian_ids,
                        segmented)
    means2d, radii, depths = _cuda(means2d, radii, depths)
    n_tiles = tile_width * tile_height
    tile_bits = floor_log2_plus_one(n_tiles)
    image_bits = floor_log2_plus_one(I)
    if sort and max(tile_width, tile_height) <= 65535:
        tiles_per_gauss, m, bins = intersect_tile_count_totals(means2d, radii, I, tile_size,
                                                               tile_width, tile_height)
        if image_bits + tile_bits > 32:
            raise RuntimeError(
                "intersect_tile_encode image id and tile id require more than 32 bits.")
        isect_ids, flatten_ids = intersect_tile_encode_binned(
            means2d, radii, depths, I, tile_size, tile_width, tile_height, m, bins)
        return {"tiles_per_gauss": tiles_per_gauss, "isect_ids": isect_ids,
                "flatten_ids": flatten_ids}
    tiles_per_gauss = intersect_tile_count(means2d, radii, I, tile_size, tile_width, tile_height)
    offsets, total = intersect_tile_offsets(tiles_per_gauss)
    m = int(total.item()) if tiles_per_gauss.numel() else 0
    if image_bits + tile_bits > 32:
        raise RuntimeError("intersect_tile_encode image id and tile id require more than 32 bits.")
    if sort:
        isect_ids, flatten_ids = intersect_tile_encode_sorted(
            means2d, radii, depths, tiles_per_gauss, I, tile_size, tile_width, tile_height, m)
    else:
        isect_ids, flatten_ids = intersect_tile_encode(means2d, radii, depths, offsets, I,
                                                       tile_size, tile_width, tile_height, m)
    return {"tiles_per_gauss": tiles_per_gauss, "isect_ids": isect_ids,
            "flatten_ids": flatten_ids}


def intersect_offset_forward(isect_ids, I, tile_width, tile_height):
    """binding.cpp:234-241 / gsplat_intersect.cpp:586-603."""
    if I <= 0 or tile_width <= 0 or tile_height <= 0:
        raise RuntimeError("intersect_offset expects positive image and tile dimensions.")
    isect_ids = _arr(isect_ids)
    if isect_ids.dtype != torch.int64:
        raise RuntimeError("intersect_offset expects int64 isect_ids.")
    isect_ids = _cuda(isect_ids)
    out = _empty((int(I), int(tile_height), int(tile_width)), torch.int32)
    check(_lib.load().gs_isect_offset(isect_ids.numel(), _ptr(isect_ids), int(I), int(tile_width),
                                      int(tile_height), _ptr(out), _stream()),
          "intersect_offset_forward")
    return out


# ---------------------------------------------------------------- rasterize


def _raster_common(means2d, conics, colors, opacities, tile_offsets, flatten_ids, masks):
    """gsplat_rasterize.cpp:47-87 and :173-183."""
    if means2d.dim() < 3 or means2d.shape[-1] != 2:
        raise RuntimeError("means2d must have shape [..., N, 2].")
    if conics.dim() != means2d.dim() or conics.shape[-1] != 3:
        raise RuntimeError("conics must have shape [..., N, 3].")
    if colors.dim() != means2d.dim() or colors.shape[-2] != means2d.shape[-2]:
        raise RuntimeError("colors must have shape [..., N, channels].")
    if opacities.dim() + 1 != means2d.dim():
        raise RuntimeError("opacities must have shape [..., N].")
    if tile_offsets.dim() < 3:
        raise RuntimeError("tile_offsets must have shape [..., tile_height, tile_width].")
    if flatten_ids.dim() != 1:
        raise RuntimeError("flatten_ids must have shape [n_isects].")
    if masks is not None and tuple(masks.shape) != tuple(tile_offsets.shape):
        raise RuntimeError("masks must have the same shape as tile_offsets.")
    N = means2d.shape[-2]
    th, tw = tile_offsets.shape[-2], tile_offsets.shape[-1]
    I = tile_offsets.numel() // (th * tw)
    if means2d.numel() // 2 != I * N:
        raise RuntimeError(
            "rasterize_to_pixels_3dgs dense path expects means2d size to equal I * N * 2.")
    ch = colors.shape[-1]
    if conics.numel() != I * N * 3 or colors.numel() != I * N * ch or opacities.numel() != I * N:
        raise RuntimeError("rasterize_to_pixels_3dgs: per-Gaussian inputs must be [I, N, ...].")
    for t in (means2d, conics, colors, opacities):
        if t.dtype != torch.float32:
            raise RuntimeError("rasterize_to_pixels_3dgs expects float32 inputs.")
    if tile_offsets.dtype != torch.int32 or flatten_ids.dtype != torch.int32:
        raise RuntimeError("rasterize_to_pixels_3dgs expects int32 tile_offsets and flatten_ids.")
    return I, N, ch, th, tw


def rasterize_to_pixels_3dgs_forward(inputs, image_width, image_height, tile_size):
    """binding.cpp:243-283 / gsplat_rasterize.cpp:165-208."""
    means2d = _req(inputs, "means2d")
    conics = _req(inputs, "conics")
    colors = _req(inputs, "colors")
    opacities = _req(inputs, "opacities")
    tile_offsets = _req(inputs, "tile_offsets")
    flatten_ids = _req(inputs, "flatten_ids")
    backgrounds = _opt(inputs, "backgrounds")
    masks = _as_bool_u8(_opt(inputs, "masks"))
    if means2d.dim() == 2:
        raise RuntimeError("rasterize_to_pixels_3dgs packed path is not implemented yet.")
    I, N, ch, th, tw = _raster_common(means2d, conics, colors, opacities, tile_offsets,
                                      flatten_ids, masks)
    if backgrounds is not None and backgrounds.numel() != I * ch:
        raise RuntimeError("backgrounds must have shape [..., channels].")
    prefix = tuple(tile_offsets.shape[:-2])
    H, W = int(image_height), int(image_width)
    means2d, conics, colors, opacities, tile_offsets, flatten_ids, backgrounds, masks = _cuda(
        means2d, conics, colors, opacities, tile_offsets, flatten_ids, backgrounds, masks)
    out = {
        "render_colors": _empty(prefix + (H, W, ch)),
        "render_alphas": _empty(prefix + (H, W, 1)),
        "last_ids": _empty(prefix + (H, W), torch.int32),
    }
    p = RasterParams(I, N, ch, W, H, int(tile_size), tw, th, flatten_ids.numel(),
                     int(backgrounds is not None), int(masks is not None), 0)
    bounds = sigma_bounds(opacities)
    p.sigma_bounds = _ptr(bounds)
    check(_lib.load().gs_rasterize_fwd(ct.byref(p), _ptr(means2d), _ptr(conics), _ptr(colors),
                                       _ptr(opacities), _ptr(backgrounds), _ptr(masks),
                                       _ptr(tile_offsets), _ptr(flatten_ids),
                                       _ptr(out["render_colors"]), _ptr(out["render_alphas"]),
                                       _ptr(out["last_ids"]), _stream()),
          "rasterize_to_pixels_3dgs_forward")
    return out


def sigma_bounds(opacities):
    """The rasterizer's exact alpha decisions as two sigma bounds per opacity
    entry ([n, 2] float32; gs_rasterize_sigma_bounds), computed once and read
    by every tile instead of being derived per staged entry."""
    o = opacities.contiguous()
    out = torch.empty((o.numel(), 2), dtype=torch.float32, device=o.device)
    check(_lib.load().gs_rasterize_sigma_bounds(o.numel(), _ptr(o), None, 0, _ptr(out),
                                                _stream()),
          "rasterize_sigma_bounds")
    return out


def rasterize_to_pixels_3dgs_backward(inputs, forward_outputs, cotangents, image_width,
                                      image_height, tile_size, absgrad=False):
    """binding.cpp:285-344 / gsplat_rasterize.cpp:210-247."""
    means2d = _req(inputs, "means2d")
    conics = _req(inputs, "conics")
    colors = _req(inputs, "colors")
    opacities = _req(inputs, "opacities")
    tile_offsets = _req(inputs, "tile_offsets")
    flatten_ids = _req(inputs, "flatten_ids")
    render_alphas = _req(forward_outputs, "render_alphas")
    last_ids = _req(forward_outputs, "last_ids")
    v_render_colors = _req(cotangents, "v_render_colors")
    v_render_alphas = _req(cotangents, "v_render_alphas")
    backgrounds = _opt(inputs, "backgrounds")
    masks = _as_bool_u8(_opt(inputs, "masks"))
    if means2d.dim() == 2:
        raise RuntimeError("rasterize_to_pixels_3dgs packed path is not implemented yet.")
    I, N, ch, th, tw = _raster_common(means2d, conics, colors, opacities, tile_offsets,
                                      flatten_ids, masks)
    H, W = int(image_height), int(image_width)
    prefix = tuple(tile_offsets.shape[:-2])
    if render_alphas.dim() < 3 or render_alphas.shape[-1] != 1:
        raise RuntimeError("render_alphas must have shape [..., H, W, 1].")
    if last_ids.dim() + 1 != render_alphas.dim():
        raise RuntimeError("last_ids must have shape [..., H, W].")
    if tuple(v_render_colors.shape) != prefix + (H, W, ch):
        raise RuntimeError("v_render_colors shape mismatch.")
    if tuple(v_render_alphas.shape) != tuple(render_alphas.shape):
        raise RuntimeError("v_render_alphas shape mismatch.")
    if render_alphas.numel() != I * H * W or last_ids.numel() != I * H * W:
        raise RuntimeError("render_alphas / last_ids must cover [I, H, W].")
    (means2d, conics, colors, opacities, tile_offsets, flatten_ids, backgrounds, masks,
     render_alphas, last_ids, v_render_colors, v_render_alphas) = _cuda(
        means2d, conics, colors, opacities, tile_offsets, flatten_ids, backgrounds, masks,
        render_alphas, last_ids, v_render_colors, v_render_alphas)
    out = {}
    if absgrad:
        out["v_means2d_abs"] = _empty(tuple(means2d.shape))
    out["v_means2d"] = _empty(tuple(means2d.shape))
    out["v_conics"] = _empty(tuple(conics.shape))
    out["v_colors"] = _empty(tuple(colors.shape))
    out["v_opacities"] = _empty(tuple(opacities.shape))
    if backgrounds is not None:
        out["v_backgrounds"] = _empty(tuple(backgrounds.shape))
    p = RasterParams(I, N, ch, W, H, int(tile_size), tw, th, flatten_ids.numel(),
                     int(backgrounds is not None), int(masks is not None), int(bool(absgrad)))
    bounds = sigma_bounds(opacities)
    p.sigma_bounds = _ptr(bounds)
    check(_lib.load().gs_rasterize_bwd(ct.byref(p), _ptr(means2d), _ptr(conics), _ptr(colors),
                                       _ptr(opacities), _ptr(backgrounds), _ptr(masks),
                                       _ptr(tile_offsets), _ptr(flatten_ids), _ptr(render_alphas),
                                       _ptr(last_ids), _ptr(v_render_colors),
                                       _ptr(v_render_alphas), _ptr(out.get("v_means2d_abs")),
                                       _ptr(out["v_means2d"]), _ptr(out["v_conics"]),
                                       _ptr(out["v_colors"]), _ptr(out["v_opacities"]),
                                       _ptr(out.get("v_backgrounds")), _stream()),
          "rasterize_to_pixels_3dgs_backward")
    return out


# ---------------------------------------------------------------- SH


def _validate_sh(degree, dirs, coeffs, masks, name):
    """gsplat_spherical_harmonics.cpp:42-110."""
    if degree < 0 or degree > 4:
        raise RuntimeError(f"{name} supports degree 0..4.")
    if dirs.dtype != torch.float32 or coeffs.dtype != torch.float32:
        raise RuntimeError(f"{name} currently supports float32 dirs and coeffs.")
    if dirs.dim() < 1 or dirs.shape[-1] != 3:
        raise RuntimeError("dirs must have shape [..., 3].")
    if coeffs.dim() < 2 or coeffs.shape[-1] != 3:
        raise RuntimeError("coeffs must have shape [..., K, 3].")
    K = coeffs.shape[-2]
    if K < (degree + 1) ** 2:
        raise RuntimeError("coeffs has fewer SH bases than degrees_to_use requires.")
    if coeffs.numel() // (K * 3) != dirs.numel() // 3:
        raise RuntimeError("dirs and coeffs prefix dimensions must have the same size.")
    if masks is not None and masks.numel() != dirs.numel() // 3:
        raise RuntimeError("masks must have shape matching dirs prefix dims.")
    return K


def spherical_harmonics_forward(degrees_to_use, inputs):
    """binding.cpp:346-362 / gsplat_spherical_harmonics.cpp:429-441."""
    dirs = _req(inputs, "dirs")
    coeffs = _req(inputs, "coeffs")
    masks = _as_bool_u8(_opt(inputs, "masks"))
    K = _validate_sh(int(degrees_to_use), dirs, coeffs, masks, "spherical_harmonics_forward")
    dirs, coeffs, masks = _cuda(dirs, coeffs, masks)
    colors = _empty(tuple(dirs.shape))
    p = SHParams(dirs.numel() // 3, K, int(degrees_to_use), int(masks is not None))
    check(_lib.load().gs_sh_fwd(ct.byref(p), _ptr(dirs), _ptr(coeffs), _ptr(masks), _ptr(colors),
                                _stream()), "spherical_harmonics_forward")
    return colors


def spherical_harmonics_backward(degrees_to_use, inputs, cotangents, compute_v_dirs=True):
    """binding.cpp:364-392 / gsplat_spherical_harmonics.cpp:443-464."""
    dirs = _req(inputs, "dirs")
    coeffs = _req(inputs, "coeffs")
    v_colors = _req(cotangents, "v_colors")
    masks = _as_bool_u8(_opt(inputs, "masks"))
    K = _validate_sh(int(degrees_to_use), dirs, coeffs, masks, "spherical_harmonics_backward")
    if v_colors.dtype != torch.float32:
        raise RuntimeError("spherical_harmonics_backward currently supports float32 arrays.")
    if tuple(v_colors.shape) != tuple(dirs.shape):
        raise RuntimeError("v_colors must have the same shape as dirs.")
    dirs, coeffs, masks, v_colors = _cuda(dirs, coeffs, masks, v_colors)
    v_coeffs = _empty(tuple(coeffs.shape))
    v_dirs = _empty(tuple(dirs.shape)) if compute_v_dirs else None
    p = SHParams(dirs.numel() // 3, K, int(degrees_to_use), int(masks is not None))
    check(_lib.load().gs_sh_bwd(ct.byref(p), _ptr(dirs), _ptr(coeffs), _ptr(masks),
                                _ptr(v_colors), _ptr(v_dirs), _ptr(v_coeffs), _stream()),
          "spherical_harmonics_backward")
    out = {}
    if compute_v_dirs:
        out["v_dirs"] = v_dirs
    out["v_coeffs"] = v_coeffs
    return out


# ---------------------------------------------------------------- quat/scale


def _validate_qs(quats, scales, name):
    """gsplat_quat_scale_to_covar.cpp:50-68."""
    if quats.dtype != torch.float32 or scales.dtype != torch.float32:
        raise RuntimeError(f"{name} currently supports float32 inputs.")
    if quats.dim() < 1 or quats.shape[-1] != 4:
        raise RuntimeError("quats must have shape [..., 4].")
    if scales.dim() < 1 or scales.shape[-1] != 3:
        raise RuntimeError("scales must have shape [..., 3].")
    if quats.numel() // 4 != scales.numel() // 3:
        raise RuntimeError("quats and scales prefix dimensions must have the same size.")


def quat_scale_to_covar_preci_forward(inputs, compute_covar=True, compute_preci=True, triu=True):
    """binding.cpp:394-416 / gsplat_quat_scale_to_covar.cpp:337-354."""
    quats = _req(inputs, "quats")
    scales = _req(inputs, "scales")
    _validate_qs(quats, scales, "quat_scale_to_covar_preci_forward")
    quats, scales = _cuda(quats, scales)
    tail = (6,) if triu else (3, 3)
    shape = tuple(quats.shape[:-1]) + tail
    covars = _empty(shape) if compute_covar else _zeros0()
    precis = _empty(shape) if compute_preci else _zeros0()
    p = QS2CParams(quats.numel() // 4, int(bool(compute_covar)), int(bool(compute_preci)),
                   int(bool(triu)))
    check(_lib.load().gs_quat_scale_to_covar_fwd(ct.byref(p), _ptr(quats), _ptr(scales),
                                                 _ptr(covars) if compute_covar else None,
                                                 _ptr(precis) if compute_preci else None,
                                                 _stream()),
          "quat_scale_to_covar_preci_forward")
    return {"covars": covars, "precis": precis}


def quat_scale_to_covar_preci_backward(inputs, cotangents, triu=True):
    """binding.cpp:418-443 / gsplat_quat_scale_to_covar.cpp:356-372."""
    quats = _req(inputs, "quats")
    scales = _req(inputs, "scales")
    v_covars = _opt(cotangents, "v_covars")
    v_precis = _opt(cotangents, "v_precis")
    _validate_qs(quats, scales, "quat_scale_to_covar_preci_backward")
    expected = tuple(quats.shape[:-1]) + ((6,) if triu else (3, 3))
    if v_covars is not None and v_covars.dtype != torch.float32:
        raise RuntimeError("v_covars must be float32.")
    if v_precis is not None and v_precis.dtype != torch.float32:
        raise RuntimeError("v_precis must be float32.")
    if v_covars is not None and tuple(v_covars.shape) != expected:
        raise RuntimeError("v_covars shape does not match triu output shape.")
    if v_precis is not None and tuple(v_precis.shape) != expected:
        raise RuntimeError("v_precis shape does not match triu output shape.")
    quats, scales, v_covars, v_precis = _cuda(quats, scales, v_covars, v_precis)
    v_quats = _empty(tuple(quats.shape))
    v_scales = _empty(tuple(scales.shape))
    n = quats.numel() // 4
    # With neither cotangent the kernel writes zero gradients (the reference
    # zero-fills its outputs).
    p = QS2CParams(n, int(v_covars is not None), int(v_precis is not None), int(bool(triu)))
    check(_lib.load().gs_quat_scale_to_covar_bwd(ct.byref(p), _ptr(quats), _ptr(scales),
                                                 _ptr(v_covars), _ptr(v_precis), _ptr(v_quats),
                                                 _ptr(v_scales), _stream()),
          "quat_scale_to_covar_preci_backward")
    return {"v_quats": v_quats, "v_scales": v_scales}
