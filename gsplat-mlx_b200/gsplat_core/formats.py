"""On-disk formats of the reference trainer around the hot path
(scripts/test/scanner_points_training_utils.py):

* ``spz_attributes`` -- the arrays export_trained_spz (:1424-1493) hands to the
  spz package's GaussianCloud, computed on device by gs_spz_attributes
  (positions in the SPZ axes, scales, rotations through the chosen axis
  convention and storage order, alphas, colours, SH rest coefficients).
  Writing the .spz file itself is the third-party spz package's work
  (spz.save_spz packs and gzips the arrays); ``write_spz`` calls it when it
  is importable, as the reference does, and raises ImportError otherwise.
* ``save_checkpoint_npz`` / ``load_checkpoint_npz`` -- the parameter
  checkpoint of save_model_parameters_npz (:1608-1651): the same keys,
  dtypes and shapes (a leading batch axis of 1), compressed npz.
"""
from __future__ import annotations

import ctypes as ct
import json
import os

import numpy as np
import torch

from . import _lib
from ._lib import SpzParams, check

SCALE_MODES = {"direct": 0, "scanner_axis": 1}
ROTATION_MODES = {"direct": 0, "position_axis": 1, "fastgs_conjugate": 2,
                  "position_conjugate": 3}
QUAT_ORDERS = {"wxyz": 0, "xyzw": 1}
COLOR_MODES = {"sh": 0, "raw_rgb": 1}


def _p(t):
    return None if t is None else ct.c_void_p(t.data_ptr())


def _mode(table, value, what):
    if value not in table:
        raise ValueError(f"Unsupported SPZ {what}: {value}")
    return table[value]


def spz_attributes(means, quats, log_scales, opacity_logits, features_dc=None,
                   features_rest=None, colors=None, sh_degree=0, scale_mode="direct",
                   rotation_mode="direct", quat_order="wxyz", color_mode="sh"):
    """Device fp32 tensors [N, ...] of one model (no batch axis): an SH model
    gives ``features_dc`` [N,3] and ``features_rest`` [N,K-1,3]; an RGB model
    gives ``colors`` [N,3] (its activated colours).  Returns
    {"positions", "scales", "rotations", "alphas", "colors", "sh",
    "sh_degree"} as flat fp32 device tensors, the GaussianCloud fields."""
    n = means.shape[0]
    rgb = colors is not None
    if rgb == (features_dc is not None):
        raise ValueError("spz_attributes: give features_dc (SH model) or colors (RGB model)")
    cm = _mode(COLOR_MODES, color_mode, "color mode")
    rest = (int(sh_degree) + 1) ** 2 - 1 if (not rgb and cm == 0) else 0
    stride = features_rest.shape[-2] if (features_rest is not None and features_rest.dim() == 3) else 0
    if rest > stride:
        raise ValueError(f"spz_attributes: SH degree {sh_degree} needs {rest} rest coefficients, "
                         f"features_rest has {stride}")
    src = (colors if rgb else features_dc).contiguous()
    ins = [t.contiguous() for t in (means, quats, log_scales, opacity_logits)]
    dev = means.device
    e = lambda *shape: torch.empty(shape, dtype=torch.float32, device=dev)  # noqa: E731
    out = {"positions": e(n, 3), "scales": e(n, 3), "rotations": e(n, 4), "alphas": e(n),
           "colors": e(n, 3), "sh": e(n, rest, 3) if rest else e(0)}
    p = SpzParams(n, _mode(SCALE_MODES, scale_mode, "scale mode"),
                  _mode(ROTATION_MODES, rotation_mode, "rotation mode"),
                  _mode(QUAT_ORDERS, quat_order, "quaternion order"), cm, int(rgb), rest, stride)
    fr = features_rest.contiguous() if rest else None
    check(_lib.load().gs_spz_attributes(
        ct.byref(p), *[_p(t) for t in ins], _p(src), _p(fr), _p(out["positions"]),
        _p(out["scales"]), _p(out["rotations"]), _p(out["alphas"]), _p(out["colors"]),
        _p(out["sh"]) if rest else None,
        ct.c_void_p(torch.cuda.current_stream(dev).cuda_stream)), "spz_attributes")
    out = {k: v.reshape(-1) for k, v in out.items()}
    out["sh_degree"] = int(sh_degree) if rest else 0
    return out


def write_spz(path, attributes, antialiased=True):
    """Writes the attributes with the spz package (spz.GaussianCloud +
    spz.save_spz), the way export_trained_spz does; returns the Gaussian
    count.  Raises ImportError when the package is not installed."""
    try:
        import spz
    except ImportError as exc:
        raise ImportError("The 'spz' Python package is required for SPZ export.") from exc
    cloud = spz.GaussianCloud()
    cloud.antialiased = antialiased
    for k in ("positions", "scales", "rotations", "alphas", "colors", "sh"):
        setattr(cloud, k, attributes[k].detach().cpu().numpy().astype(np.float32))
    cloud.sh_degree = int(attributes["sh_degree"])
    os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
    if not spz.save_spz(cloud, spz.PackOptions(), str(path)):
        raise RuntimeError(f"failed to save spz to {path}")
    return int(attributes["positions"].numel() // 3)


def _host(t):
    return np.asarray(t.detach().cpu().numpy() if isinstance(t, torch.Tensor) else t, np.float32)


def save_checkpoint_npz(path, means, quats, log_scales, opacity_logits, features_dc=None,
                        features_rest=None, color_logits=None, active_sh_degree=0,
                        max_sh_degree=0, summary=None):
    """save_model_parameters_npz: [N, ...] tensors (an SH model's
    features_dc / features_rest, or an RGB model's color_logits) are stored
    with the reference's leading batch axis; quats are stored normalised
    (``quats_wxyz``, the model's normalized_quats)."""
    q = _host(quats)
    q = q / np.maximum(np.sqrt(np.sum(q * q, axis=-1, keepdims=True)), np.float32(1e-8))
    rgb = color_logits is not None
    payload = {"color_mode": np.array("rgb" if rgb else "sh", dtype=np.str_),
               "active_sh_degree": np.array(active_sh_degree, dtype=np.int32),
               "max_sh_degree": np.array(max_sh_degree, dtype=np.int32),
               "means": _host(means)[None], "quats_wxyz": q[None],
               "log_scales": _host(log_scales)[None]}
    if rgb:
        payload["color_logits"] = _host(color_logits)[None, None]
    else:
        payload["features_dc"] = _host(features_dc)[None]
        payload["features_rest"] = _host(features_rest)[None]
    payload["opacity_logits"] = _host(opacity_logits)[None]
    payload["summary_json"] = np.array(json.dumps(summary or {}), dtype=np.str_)
    os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
    np.savez_compressed(path, **payload)


def load_checkpoint_npz(path, device=None):
    """The arrays of a save_model_parameters_npz checkpoint without the batch
    axis, as fp32 tensors on ``device`` (host when None), plus color_mode,
    the SH degrees and the summary dict."""
    d = np.load(path)
    out = {"color_mode": str(d["color_mode"]), "active_sh_degree": int(d["active_sh_degree"]),
           "max_sh_degree": int(d["max_sh_degree"]), "summary": json.loads(str(d["summary_json"]))}
    for k in ("means", "quats_wxyz", "log_scales", "features_dc", "features_rest",
              "opacity_logits"):
        if k in d:
            out[k] = torch.from_numpy(np.ascontiguousarray(d[k][0])).to(device or "cpu")
    if "color_logits" in d:
        out["color_logits"] = torch.from_numpy(np.ascontiguousarray(d["color_logits"][0, 0])).to(
            device or "cpu")
    return out
