"""CPU restatement of the reference trainer's export conversions (TEST
INFRASTRUCTURE ONLY: tests/ use it as the checker of gs_spz_attributes; the
product never imports it).

Follows scripts/test/scanner_points_training_utils.py: positions_to_spz
(:1361-1366), scales_to_spz (:1380-1389), quat_wxyz_to_rotmat (:1311-1324),
rotmat_to_quat_wxyz (:1327-1358, Shepperd's method with the reference's
branch order), quats_to_spz (:1392-1412), quats_to_spz_storage (:1415-1421)
and the colour / SH selection of export_trained_spz (:1461-1486), in numpy
fp32.  Pinned against tests/golden/formats.npz, which the reference's own
export_trained_spz produced (tests/golden/make_formats_golden.py).
"""
from __future__ import annotations

import numpy as np

SH_C0 = 0.28209479177387814
_POSITION_AXIS = np.array([[1, 0, 0], [0, 0, -1], [0, 1, 0]], np.float32)
_FASTGS_AXIS = np.array([[1, 0, 0], [0, 0, 1], [0, -1, 0]], np.float32)


def _normalize(q):
    return q / np.clip(np.linalg.norm(q, axis=1, keepdims=True), 1.0e-8, None)


def _rotmat(q):
    q = _normalize(q)
    w, x, y, z = q[:, 0], q[:, 1], q[:, 2], q[:, 3]
    r = np.empty((q.shape[0], 3, 3), np.float32)
    r[:, 0] = np.stack([1 - 2 * (y * y + z * z), 2 * (x * y - z * w), 2 * (x * z + y * w)], -1)
    r[:, 1] = np.stack([2 * (x * y + z * w), 1 - 2 * (x * x + z * z), 2 * (y * z - x * w)], -1)
    r[:, 2] = np.stack([2 * (x * z - y * w), 2 * (y * z + x * w), 1 - 2 * (x * x + y * y)], -1)
    return r


def _quat(r):
    """Largest-of-four quaternion extraction, branches in the reference's
    order: trace > 0, then r00 the largest diagonal entry, then r11 > r22."""
    q = np.empty((r.shape[0], 4), np.float32)
    tr = r[:, 0, 0] + r[:, 1, 1] + r[:, 2, 2]
    b0 = tr > 0
    b1 = ~b0 & (r[:, 0, 0] > r[:, 1, 1]) & (r[:, 0, 0] > r[:, 2, 2])
    b2 = ~b0 & ~b1 & (r[:, 1, 1] > r[:, 2, 2])
    b3 = ~b0 & ~b1 & ~b2
    for m, diag, comps in (
            (b0, None, lambda m, s: [0.25 * s, (r[m, 2, 1] - r[m, 1, 2]) / s,
                                     (r[m, 0, 2] - r[m, 2, 0]) / s, (r[m, 1, 0] - r[m, 0, 1]) / s]),
            (b1, 0, lambda m, s: [(r[m, 2, 1] - r[m, 1, 2]) / s, 0.25 * s,
                                  (r[m, 0, 1] + r[m, 1, 0]) / s, (r[m, 0, 2] + r[m, 2, 0]) / s]),
            (b2, 1, lambda m, s: [(r[m, 0, 2] - r[m, 2, 0]) / s, (r[m, 0, 1] + r[m, 1, 0]) / s,
                                  0.25 * s, (r[m, 1, 2] + r[m, 2, 1]) / s]),
            (b3, 2, lambda m, s: [(r[m, 1, 0] - r[m, 0, 1]) / s, (r[m, 0, 2] + r[m, 2, 0]) / s,
                                  (r[m, 1, 2] + r[m, 2, 1]) / s, 0.25 * s])):
        if not m.any():
            continue
        if diag is None:
            s = np.sqrt(tr[m] + 1.0) * 2.0
        else:
            o = [i for i in range(3) if i != diag]
            s = np.sqrt(1.0 + r[m, diag, diag] - r[m, o[0], o[0]] - r[m, o[1], o[1]]) * 2.0
        q[m] = np.stack(comps(m, s), -1)
    return _normalize(q)


def spz_attributes(means, quats, log_scales, opacity_logits, colors_or_dc, features_rest=None,
                   scale_mode="direct", rotation_mode="direct", quat_order="wxyz",
                   color_mode="sh", source="sh", sh_degree=3):
    """The arrays export_trained_spz hands to spz.GaussianCloud, [N, ...]:
    positions, scales, rotations, alphas, colors, sh (and the SH degree).
    source "sh": colors_or_dc = features_dc [N,3], features_rest [N,K-1,3];
    source "rgb": colors_or_dc = the model's colours (sigmoid of its logits)."""
    p = np.stack([means[:, 0], -means[:, 2], means[:, 1]], -1).astype(np.float32)
    s = log_scales.astype(np.float32) if scale_mode == "direct" else \
        log_scales[:, [0, 2, 1]].astype(np.float32)
    if rotation_mode == "direct":
        q = _normalize(quats)
    else:
        r = _rotmat(quats)
        if rotation_mode == "position_axis":
            r = _POSITION_AXIS @ r
        elif rotation_mode == "fastgs_conjugate":
            r = _FASTGS_AXIS @ r @ _FASTGS_AXIS.T
        else:
            r = _POSITION_AXIS @ r @ _POSITION_AXIS.T
        q = _quat(r)
    q = _normalize(q)
    if quat_order == "xyzw":
        q = q[:, [1, 2, 3, 0]]
    out = {"positions": p, "scales": s, "rotations": q.astype(np.float32),
           "alphas": opacity_logits.astype(np.float32)}
    c = np.asarray(colors_or_dc, np.float32)
    if source == "rgb":
        out["colors"] = (np.clip(c, 0, 1) - 0.5) / SH_C0 if color_mode == "sh" else np.clip(c, 0, 1)
        out["sh"], out["sh_degree"] = np.zeros((0,), np.float32), 0
    elif color_mode == "sh":
        rest = (sh_degree + 1) ** 2 - 1
        out["colors"], out["sh"] = c, features_rest[:, :rest, :]
        out["sh_degree"] = sh_degree
    else:
        out["colors"] = np.clip(0.5 + SH_C0 * c, 0, 1)
        out["sh"], out["sh_degree"] = np.zeros((0,), np.float32), 0
    out["colors"] = out["colors"].astype(np.float32)
    return out
