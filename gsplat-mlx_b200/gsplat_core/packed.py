"""Packed [nnz] layout: only the visible (camera, Gaussian) entries, as rows
in (image, Gaussian) order, through intersection and rasterization -- the
upstream-gsplat form the reference refuses ("intersect_tile packed path is
not implemented yet", gsplat_intersect.cpp:115-118).  With many cameras most
(camera, Gaussian) entries are culled, and the element passes of the
intersection then run over the visible rows only.

    packed = pack_projection(projection_ewa_3dgs_fused_forward(...))
    isect = intersect_tile_packed_forward(packed, I, tile_size, tw, th)
    out = rasterize_packed_forward(packed_inputs, isect, I, W, H, tile_size)

The rows are exactly the dense outputs' visible entries; the sorted lists
are the dense lists with element ids replaced by row ids, so renders and
gradients equal the dense path's.  ``unpack_rows`` scatters per-row
gradients back to the dense [I, N, ...] layout of the projection backward.
"""
from __future__ import annotations

import ctypes as ct

import torch

from . import _lib
from ._lib import IsectParams, RasterParams, check


def _p(t):
    return None if t is None else ct.c_void_p(t.data_ptr())


def _s():
    return ct.c_void_p(torch.cuda.current_stream().cuda_stream)


def pack_projection(proj):
    """Packed rows of a dense projection output (radii [..., N, 2], means2d,
    depths, conics, compensations [..., N] or [0]): {"image_ids",
    "gaussian_ids", "radii", "means2d", "depths", "conics", "compensations"
    (or None)} with nnz rows, image = flattened leading index."""
    radii = proj["radii"].contiguous()
    N = radii.shape[-2]
    n = radii.numel() // 2
    comps = proj.get("compensations")
    comps = comps.contiguous() if comps is not None and comps.numel() else None
    m2, dep, con = (proj[k].contiguous() for k in ("means2d", "depths", "conics"))
    lib = _lib.load()
    dev = radii.device
    ws = torch.empty((lib.gs_pack_visible_workspace_size(n),), dtype=torch.uint8, device=dev)
    nnz_dev = torch.zeros((1,), dtype=torch.int64, device=dev)

    def call(cap, o):
        check(lib.gs_pack_visible(n, max(N, 1), _p(radii), _p(m2), _p(dep), _p(con), _p(comps),
                                  cap, *(_p(o.get(k)) for k in (
                                      "image_ids", "gaussian_ids", "radii", "means2d", "depths",
                                      "conics", "compensations")),
                                  _p(nnz_dev), _p(ws), ws.numel(), _s()), "pack_projection")

    call(0, {})
    nnz = int(nnz_dev.item())
    i32 = lambda *s: torch.empty(s, dtype=torch.int32, device=dev)  # noqa: E731
    f32 = lambda *s: torch.empty(s, dtype=torch.float32, device=dev)  # noqa: E731
    out = {"image_ids": i32(nnz), "gaussian_ids": i32(nnz), "radii": i32(nnz, 2),
           "means2d": f32(nnz, 2), "depths": f32(nnz), "conics": f32(nnz, 3),
           "compensations": f32(nnz) if comps is not None else None}
    call(nnz, out)
    return out


def intersect_tile_packed_forward(packed, I, tile_size, tile_width, tile_height):
    """Sorted intersections of packed rows (image_ids in [0, I)): the same
    keys as the dense intersect_tile_forward(sort=True), flatten_ids = row
    ids, plus the tile offsets [I, tile_height, tile_width]."""
    ids = packed["image_ids"]
    nnz = ids.numel()
    if nnz and (int(ids.min()) < 0 or int(ids.max()) >= int(I)):
        raise RuntimeError(f"intersect_tile_packed_forward: image ids outside [0, {I}).")
    if max(tile_width, tile_height) > 65535:
        raise RuntimeError("intersect_tile_packed_forward: more than 65535 tiles per row or column.")
    lib = _lib.load()
    dev = ids.device
    m2, radii, dep = (packed[k].contiguous() for k in ("means2d", "radii", "depths"))
    totals = torch.zeros((2,), dtype=torch.int64, device=dev)
    tpg = torch.empty((max(nnz, 1),), dtype=torch.int32, device=dev)
    cp = IsectParams(1, nnz, int(tile_size), int(tile_width), int(tile_height))
    check(lib.gs_isect_tile_count_totals(ct.byref(cp), _p(m2), _p(radii), _p(tpg), _p(totals),
                                         _s()), "intersect_tile_packed_forward")
    m, bins = (int(v) for v in totals.tolist())
    if m >= 2 ** 31:
        raise RuntimeError(f"intersect_tile_encode: {m} intersections exceed the int32 index range")
    p = IsectParams(int(I), nnz, int(tile_size), int(tile_width), int(tile_height))
    ws = torch.empty((max(1, lib.gs_isect_tile_encode_binned_packed_workspace_size(
        ct.byref(p), bins)),), dtype=torch.uint8, device=dev)
    isect_ids = torch.empty((m,), dtype=torch.int64, device=dev)
    flatten_ids = torch.empty((m,), dtype=torch.int32, device=dev)
    offsets = torch.empty((int(I), int(tile_height), int(tile_width)), dtype=torch.int32,
                          device=dev)
    check(lib.gs_isect_tile_encode_binned_packed(
        ct.byref(p), _p(ids.contiguous()), _p(m2), _p(radii), _p(dep), m, bins, _p(isect_ids),
        _p(flatten_ids), _p(offsets), _p(ws), ws.numel(), _s()), "intersect_tile_packed_forward")
    if bins > 0:
        check(lib.gs_isect_tile_encode_binned_check(bins, _p(ws), _s()),
              "intersect_tile_packed_forward")
    return {"isect_ids": isect_ids, "flatten_ids": flatten_ids, "tile_offsets": offsets}


def _raster_params(inputs, isect, I, W, H, ts, absgrad=False):
    ch = inputs["colors"].shape[-1]
    th, tw = isect["tile_offsets"].shape[-2:]
    bg = inputs.get("backgrounds")
    masks = inputs.get("masks")
    # N = 0: the rows are packed, nothing is sized by I * N
    return RasterParams(int(I), 0, ch, int(W), int(H), int(ts), tw, th,
                        isect["flatten_ids"].numel(), int(bg is not None),
                        int(masks is not None), int(bool(absgrad))), ch, bg, masks


def rasterize_packed_forward(inputs, isect, I, image_width, image_height, tile_size):
    """inputs: means2d [nnz,2], conics [nnz,3], colors [nnz,ch], opacities
    [nnz], optional backgrounds [I,ch] and masks [I,th,tw] (bool).  Returns
    render_colors [I,H,W,ch], render_alphas [I,H,W,1], last_ids [I,H,W]."""
    p, ch, bg, masks = _raster_params(inputs, isect, I, image_width, image_height, tile_size)
    dev = inputs["means2d"].device
    H, W = int(image_height), int(image_width)
    out = {"render_colors": torch.empty((I, H, W, ch), dtype=torch.float32, device=dev),
           "render_alphas": torch.empty((I, H, W, 1), dtype=torch.float32, device=dev),
           "last_ids": torch.empty((I, H, W), dtype=torch.int32, device=dev)}
    m = masks.to(torch.uint8).contiguous() if masks is not None else None
    check(_lib.load().gs_rasterize_fwd(
        ct.byref(p), *(_p(inputs[k].contiguous()) for k in ("means2d", "conics", "colors",
                                                             "opacities")),
        _p(bg.contiguous() if bg is not None else None), _p(m), _p(isect["tile_offsets"]),
        _p(isect["flatten_ids"]), _p(out["render_colors"]), _p(out["render_alphas"]),
        _p(out["last_ids"]), _s()), "rasterize_packed_forward")
    return out


def rasterize_packed_backward(inputs, isect, forward_outputs, cotangents, I, image_width,
                              image_height, tile_size, absgrad=False):
    """Per-row gradients v_means2d [nnz,2], v_conics, v_colors, v_opacities
    (+ v_means2d_abs, v_backgrounds)."""
    p, ch, bg, masks = _raster_params(inputs, isect, I, image_width, image_height, tile_size,
                                      absgrad)
    p.accumulate = 1  # the row gradients are zeroed here, not sized by I * N
    z = lambda t: torch.zeros_like(t, dtype=torch.float32)  # noqa: E731
    out = {"v_means2d": z(inputs["means2d"]), "v_conics": z(inputs["conics"]),
           "v_colors": z(inputs["colors"]), "v_opacities": z(inputs["opacities"])}
    if absgrad:
        out["v_means2d_abs"] = z(inputs["means2d"])
    if bg is not None:
        out["v_backgrounds"] = z(bg)
    m = masks.to(torch.uint8).contiguous() if masks is not None else None
    check(_lib.load().gs_rasterize_bwd(
        ct.byref(p), *(_p(inputs[k].contiguous()) for k in ("means2d", "conics", "colors",
                                                             "opacities")),
        _p(bg.contiguous() if bg is not None else None), _p(m), _p(isect["tile_offsets"]),
        _p(isect["flatten_ids"]), _p(forward_outputs["render_alphas"]),
        _p(forward_outputs["last_ids"]), _p(cotangents["v_render_colors"].contiguous()),
        _p(cotangents["v_render_alphas"].contiguous()), _p(out.get("v_means2d_abs")),
        _p(out["v_means2d"]), _p(out["v_conics"]), _p(out["v_colors"]), _p(out["v_opacities"]),
        _p(out.get("v_backgrounds")), _s()), "rasterize_packed_backward")
    return out


def unpack_rows(values, packed, I, N):
    """Per-row values [nnz, ...] scattered into the dense [I, N, ...] layout
    (zeros at the culled entries), e.g. for the projection backward."""
    dense = torch.zeros((int(I), int(N)) + tuple(values.shape[1:]), dtype=values.dtype,
                        device=values.device)
    dense[packed["image_ids"].long(), packed["gaussian_ids"].long()] = values
    return dense
