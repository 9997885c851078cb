"""CPU restatement of the reference trainer's densification statistics
(TEST INFRASTRUCTURE ONLY: tests/ use it as the checker of
gs_densify_accumulate / gs_densify_masks; the product never imports it).

Follows scripts/test/scanner_points_training_utils.py,
ScannerDefaultStrategyRuntime: update_state (:412-451), the clone selection
of _duplicate_high_grad_small (:556-569), the split mask of
_split_high_grad_large (:639-657) and the prune mask of _prune_gaussians
(:706-718), with numpy's fp32 arithmetic.  Pinned against
tests/golden/densify.npz, which the reference's own class produced
(tests/golden/make_densify_golden.py).
"""
from __future__ import annotations

import numpy as np


def accumulate(v_means2d, radii, width, height, n_cameras, grad2d, count, max_radii=None):
    """One update_state call on [C, N, 2] inputs, in place on the [N]
    statistics.  Per camera in order: the scaled gradient norm of every
    visible (both radii > 0) Gaussian is added to grad2d, 1 to count; the
    normalised larger radius of the last camera that sees a Gaussian is
    max-ed into max_radii (the reference assigns through a fancy index, so
    of repeated Gaussian ids only the last write lands)."""
    v = np.array(v_means2d, np.float32, copy=True)
    r = np.asarray(radii, np.float32)
    # fp32 multiply by the Python-float scale rounded to fp32
    v[..., 0] *= np.float32(float(width) / 2.0 * float(n_cameras))
    v[..., 1] *= np.float32(float(height) / 2.0 * float(n_cameras))
    vis = (r[..., 0] > 0) & (r[..., 1] > 0)
    norms = np.sqrt(v[..., 0] * v[..., 0] + v[..., 1] * v[..., 1])
    extent = np.float32(max(width, height))
    for c in range(v.shape[0]):
        ids = np.nonzero(vis[c])[0]
        grad2d[ids] += norms[c, ids]
        count[ids] += np.float32(1.0)
    if max_radii is not None:
        last = np.full(grad2d.shape, -1.0, np.float32)
        for c in range(v.shape[0]):
            ids = np.nonzero(vis[c])[0]
            last[ids] = np.maximum(r[c, ids, 0], r[c, ids, 1]) / extent
        seen = last >= 0
        max_radii[seen] = np.maximum(max_radii[seen], last[seen])


def masks(grad2d, count, max_radii, log_scales, opacity_logits, step, n_original, cfg,
          grow=True, prune=True):
    """clone / split / prune masks (bool [n]) of one refine step and the
    prune breakdown (opacity, scale3d, scale2d, total).  cfg: the strategy
    config's fields (grow_grad2d, grow_scale3d, grow_scale2d, prune_opa,
    prune_scale3d, prune_scale2d, scene_scale, refine_scale2d_stop_iter,
    reset_every)."""
    n = log_scales.shape[0]
    out = {}
    radii_on = cfg["refine_scale2d_stop_iter"] > 0 and step < cfg["refine_scale2d_stop_iter"]
    max_scale = np.exp(np.asarray(log_scales, np.float32)).max(axis=-1)
    if grow:
        vis = count > 0
        avg = np.zeros_like(grad2d)
        avg[vis] = grad2d[vis] / np.maximum(count[vis], np.float32(1.0))
        hot = avg > np.float32(cfg["grow_grad2d"])
        lim = np.float32(cfg["grow_scale3d"] * cfg["scene_scale"])
        out["clone"] = hot & (max_scale <= lim)
        split = hot & (max_scale > lim)
        if radii_on:
            split |= max_radii > np.float32(cfg["grow_scale2d"])
        split[int(n_original):] = False
        out["split"] = split
    if prune:
        o = np.float32(1.0) / (np.float32(1.0) + np.exp(-np.asarray(opacity_logits, np.float32)))
        po = o < np.float32(cfg["prune_opa"])
        p3 = np.zeros(n, bool)
        p2 = np.zeros(n, bool)
        if step > cfg["reset_every"]:
            p3 = max_scale > np.float32(cfg["prune_scale3d"] * cfg["scene_scale"])
            if radii_on:
                p2 = max_radii > np.float32(cfg["prune_scale2d"])
        out["prune"] = po | p3 | p2
        out["prune_breakdown"] = np.array([po.sum(), p3.sum(), p2.sum(), out["prune"].sum()],
                                          np.int64)
    return out
