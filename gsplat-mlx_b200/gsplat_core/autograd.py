"""Reverse-mode wiring of the operators, the counterpart of the reference
Primitives' ``vjp`` methods, as ``torch.autograd.Function`` s.

* ``quat_scale_to_covar_preci`` -- GSPlatQuatScaleToCovarPreci::vjp
  (gsplat_quat_scale_to_covar.cpp:582-613): gradients for quats and scales.
* ``projection_ewa_3dgs_fused`` -- GSPlatProjectionEWA3DGSFused::vjp
  (gsplat_projection.cpp:1130-1208): means, covars or quats+scales, viewmats
  (only when it requires grad: viewmats_requires_grad), zero for opacities
  and Ks, and the cotangent of means2d passed unchanged to
  ``viewspace_points`` (the trainers' means2d-gradient proxy, :1200-1201).
* ``spherical_harmonics`` -- GSPlatSphericalHarmonics::vjp
  (gsplat_spherical_harmonics.cpp:670-705): v_dirs only when dirs requires
  grad (compute_v_dirs), v_coeffs always.
* ``rasterize_to_pixels_3dgs`` -- GSPlatRasterizeToPixels3DGS::vjp
  (gsplat_rasterize.cpp:749-795): absgrad off, gradients for means2d,
  conics, colors, opacities and backgrounds (when given).

Every forward and backward runs the native kernels through the drop-in
functions of ``_gsplat_core``; integer outputs (radii, last_ids) are
non-differentiable.
"""
from __future__ import annotations

import torch

from . import _gsplat_core as G


def _empty_like_none(x):
    return x is None or (isinstance(x, torch.Tensor) and x.numel() == 0)


class _QuatScaleToCovarPreci(torch.autograd.Function):
    @staticmethod
    def forward(ctx, quats, scales, compute_covar, compute_preci, triu):
        out = G.quat_scale_to_covar_preci_forward({"quats": quats, "scales": scales},
                                                  compute_covar, compute_preci, triu)
        ctx.save_for_backward(quats, scales)
        ctx.flags = (compute_covar, compute_preci, triu)
        return out["covars"], out["precis"]

    @staticmethod
    def backward(ctx, v_covars, v_precis):
        quats, scales = ctx.saved_tensors
        cc, cp, triu = ctx.flags
        cot = {}
        if cc and v_covars is not None:
            cot["v_covars"] = v_covars
        if cp and v_precis is not None:
            cot["v_precis"] = v_precis
        b = G.quat_scale_to_covar_preci_backward({"quats": quats, "scales": scales}, cot, triu)
        return b["v_quats"], b["v_scales"], None, None, None


def quat_scale_to_covar_preci(quats, scales, compute_covar=True, compute_preci=True, triu=True):
    return _QuatScaleToCovarPreci.apply(quats, scales, compute_covar, compute_preci, triu)


class _ProjectionEWA3DGSFused(torch.autograd.Function):
    @staticmethod
    def forward(ctx, means, covars, quats, scales, opacities, viewmats, Ks, viewspace_points,
                width, height, eps2d, near_plane, far_plane, radius_clip, calc_compensations,
                camera_model):
        inputs = {"means": means, "viewmats": viewmats, "Ks": Ks}
        for k, v in (("covars", covars), ("quats", quats), ("scales", scales),
                     ("opacities", opacities), ("viewspace_points", viewspace_points)):
            if not _empty_like_none(v):
                inputs[k] = v
        out = G.projection_ewa_3dgs_fused_forward(inputs, width, height, eps2d, near_plane,
                                                  far_plane, radius_clip, calc_compensations,
                                                  camera_model)
        ctx.mark_non_differentiable(out["radii"])
        ctx.save_for_backward(means, covars, quats, scales, viewmats, Ks, out["radii"],
                              out["conics"], out["compensations"])
        ctx.cfg = (width, height, eps2d, calc_compensations, camera_model)
        ctx.has = tuple(not _empty_like_none(x) for x in (covars, quats, scales, opacities,
                                                          viewspace_points))
        return out["means2d"], out["depths"], out["conics"], out["compensations"], out["radii"]

    @staticmethod
    def backward(ctx, v_means2d, v_depths, v_conics, v_comp, _v_radii):
        means, covars, quats, scales, viewmats, Ks, radii, conics, comps = ctx.saved_tensors
        width, height, eps2d, calc_comp, camera_model = ctx.cfg
        has_cov, has_q, has_s, has_op, has_vsp = ctx.has
        if camera_model != 0:
            raise RuntimeError("GSPlatProjectionEWA3DGSFused vjp currently supports pinhole only.")
        zeros = torch.zeros_like
        v_means2d = zeros(conics[..., :2]) if v_means2d is None else v_means2d
        v_depths = zeros(conics[..., 0]) if v_depths is None else v_depths
        v_conics = zeros(conics) if v_conics is None else v_conics
        inputs = {"means": means, "viewmats": viewmats, "Ks": Ks}
        if has_cov:
            inputs["covars"] = covars
        else:
            inputs["quats"], inputs["scales"] = quats, scales
        fo = {"radii": radii, "conics": conics}
        cot = {"v_means2d": v_means2d.contiguous(), "v_depths": v_depths.contiguous(),
               "v_conics": v_conics.contiguous()}
        if calc_comp:
            fo["compensations"] = comps
            cot["v_compensations"] = (zeros(comps) if v_comp is None else v_comp).contiguous()
        need_view = ctx.needs_input_grad[5]
        b = G.projection_ewa_3dgs_fused_backward(inputs, fo, cot, width, height, eps2d,
                                                 camera_model, need_view)
        grads = [b["v_means"],
                 b.get("v_covars") if has_cov else None,
                 b.get("v_quats") if not has_cov and has_q else None,
                 b.get("v_scales") if not has_cov and has_s else None,
                 None,                                     # opacities: zero (cpp:1196-1197)
                 b.get("v_viewmats") if need_view else None,
                 None,                                     # Ks: zero
                 v_means2d if has_vsp else None]           # viewspace_points proxy
        return tuple(grads) + (None,) * 8


def projection_ewa_3dgs_fused(means, viewmats, Ks, width, height, covars=None, quats=None,
                              scales=None, opacities=None, viewspace_points=None, eps2d=0.3,
                              near_plane=0.01, far_plane=1.0e10, radius_clip=0.0,
                              calc_compensations=False, camera_model=0):
    """Differentiable projection; returns (means2d, depths, conics,
    compensations, radii)."""
    return _ProjectionEWA3DGSFused.apply(means, covars, quats, scales, opacities, viewmats, Ks,
                                         viewspace_points, int(width), int(height), float(eps2d),
                                         float(near_plane), float(far_plane), float(radius_clip),
                                         bool(calc_compensations), int(camera_model))


class _SphericalHarmonics(torch.autograd.Function):
    @staticmethod
    def forward(ctx, dirs, coeffs, masks, degree):
        inputs = {"dirs": dirs, "coeffs": coeffs}
        if not _empty_like_none(masks):
            inputs["masks"] = masks
        colors = G.spherical_harmonics_forward(degree, inputs)
        ctx.save_for_backward(dirs, coeffs, masks if masks is not None else dirs.new_zeros(0))
        ctx.degree = degree
        return colors

    @staticmethod
    def backward(ctx, v_colors):
        dirs, coeffs, masks = ctx.saved_tensors
        inputs = {"dirs": dirs, "coeffs": coeffs}
        if masks.numel():
            inputs["masks"] = masks
        want_dirs = ctx.needs_input_grad[0]
        b = G.spherical_harmonics_backward(ctx.degree, inputs, {"v_colors": v_colors.contiguous()},
                                           compute_v_dirs=want_dirs)
        return (b["v_dirs"] if want_dirs else None), b["v_coeffs"], None, None


def spherical_harmonics(degrees_to_use, dirs, coeffs, masks=None):
    return _SphericalHarmonics.apply(dirs, coeffs, masks, int(degrees_to_use))


class _RasterizeToPixels3DGS(torch.autograd.Function):
    @staticmethod
    def forward(ctx, means2d, conics, colors, opacities, backgrounds, masks, tile_offsets,
                flatten_ids, width, height, tile_size):
        inputs = {"means2d": means2d, "conics": conics, "colors": colors, "opacities": opacities,
                  "tile_offsets": tile_offsets, "flatten_ids": flatten_ids}
        if not _empty_like_none(backgrounds):
            inputs["backgrounds"] = backgrounds
        if not _empty_like_none(masks):
            inputs["masks"] = masks
        out = G.rasterize_to_pixels_3dgs_forward(inputs, width, height, tile_size)
        ctx.mark_non_differentiable(out["last_ids"])
        ctx.inputs = inputs
        ctx.save_for_backward(out["render_alphas"], out["last_ids"])
        ctx.cfg = (width, height, tile_size, not _empty_like_none(backgrounds))
        ctx.rc_shape = tuple(out["render_colors"].shape)
        return out["render_colors"], out["render_alphas"], out["last_ids"]

    @staticmethod
    def backward(ctx, v_colors, v_alphas, _v_last):
        render_alphas, last_ids = ctx.saved_tensors
        width, height, tile_size, has_bg = ctx.cfg
        if v_colors is None:
            v_colors = render_alphas.new_zeros(ctx.rc_shape)
        if v_alphas is None:
            v_alphas = torch.zeros_like(render_alphas)
        b = G.rasterize_to_pixels_3dgs_backward(
            ctx.inputs, {"render_alphas": render_alphas, "last_ids": last_ids},
            {"v_render_colors": v_colors.contiguous(), "v_render_alphas": v_alphas.contiguous()},
            width, height, tile_size, absgrad=False)
        ctx.inputs = None
        return (b["v_means2d"], b["v_conics"], b["v_colors"], b["v_opacities"],
                b.get("v_backgrounds") if has_bg else None, None, None, None, None, None, None)


def rasterize_to_pixels_3dgs(means2d, conics, colors, opacities, tile_offsets, flatten_ids,
                             width, height, tile_size, backgrounds=None, masks=None):
    """Differentiable rasterization; returns (render_colors, render_alphas,
    last_ids)."""
    return _RasterizeToPixels3DGS.apply(means2d, conics, colors, opacities, backgrounds, masks,
                                        tile_offsets, flatten_ids, int(width), int(height),
                                        int(tile_size))
