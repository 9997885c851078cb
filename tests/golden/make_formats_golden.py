"""Generate tests/golden/formats.npz and tests/golden/checkpoint_sh.npz from
the reference trainer's own export code (scripts/test/
scanner_points_training_utils.py), run in this container:

* export_trained_spz (:1424-1493) for every scale / rotation / quaternion
  order / colour mode, with the SH model and the RGB model.  The reference
  hands its converted arrays to the third-party `spz` package
  (spz.GaussianCloud + spz.save_spz, which packs and gzips them); that package
  is not installed here, so a stand-in records the GaussianCloud fields the
  reference sets instead of packing them;
* save_model_parameters_npz (:1608-1651) for an SH model, written as the
  reference writes it (checkpoint_sh.npz).

MLX and the other imports of the module are replaced by numpy stand-ins, as
in make_densify_golden.py.

    python tests/golden/make_formats_golden.py [path to the reference's scripts/test]
"""
from __future__ import annotations

import itertools
import os
import sys
import types
from pathlib import Path

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from make_densify_golden import _install_stand_ins  # noqa: E402


class _Cloud:
    """The fields the reference sets on spz.GaussianCloud."""


def _install_spz(record):
    spz = types.ModuleType("spz")
    spz.GaussianCloud = _Cloud
    spz.PackOptions = lambda: None

    def save_spz(cloud, opts, path):
        record.append(cloud)
        return True

    spz.save_spz = save_spz
    sys.modules["spz"] = spz


class _SHModel:
    def __init__(self, means, quats, log_scales, dc, rest, opacity_logits):
        self.means, self.quats, self.log_scales = means[None], quats[None], log_scales[None]
        self.features_dc, self.features_rest = dc[None], rest[None]
        self.opacity_logits = opacity_logits[None]

    @property
    def normalized_quats(self):
        q = self.quats
        return q / np.maximum(np.sqrt(np.sum(q * q, axis=-1, keepdims=True)), 1e-8)


class _RGBModel(_SHModel):
    def __init__(self, means, quats, log_scales, color_logits, opacity_logits):
        self.means, self.quats, self.log_scales = means[None], quats[None], log_scales[None]
        self.color_logits = color_logits[None, None]
        self.opacity_logits = opacity_logits[None]

    @property
    def colors(self):
        return 1.0 / (1.0 + np.exp(-self.color_logits))


def main(ref_dir):
    _install_stand_ins()
    record = []
    _install_spz(record)
    sys.path.insert(0, ref_dir)
    import scanner_points_training_utils as R  # the reference module, unchanged

    rng = np.random.default_rng(11)
    N, deg, K = 64, 3, 16
    means = rng.normal(size=(N, 3)).astype(np.float32)
    quats = rng.normal(size=(N, 4)).astype(np.float32)
    quats[:8] = [[1, 0, 0, 0], [0, 1, 0, 0], [0, 0, 1, 0], [0, 0, 0, 1],
                 [-1, 0, 0, 0], [0.5, 0.5, 0.5, 0.5], [0, 0, 0.6, -0.8], [0.1, -0.7, 0.7, 0.1]]
    log_scales = rng.uniform(-6, -1, size=(N, 3)).astype(np.float32)
    dc = rng.normal(size=(N, 3)).astype(np.float32)
    rest = (0.2 * rng.normal(size=(N, K - 1, 3))).astype(np.float32)
    opacity_logits = rng.uniform(-6, 6, size=(N,)).astype(np.float32)
    color_logits = rng.normal(scale=2.0, size=(N, 3)).astype(np.float32)
    sh_model = _SHModel(means, quats, log_scales, dc, rest, opacity_logits)
    rgb_model = _RGBModel(means, quats, log_scales, color_logits, opacity_logits)

    out = dict(means=means, quats=quats, log_scales=log_scales, features_dc=dc,
               features_rest=rest, opacity_logits=opacity_logits, color_logits=color_logits,
               sh_degree=deg)
    cases = []
    for scale, rot, order, color, src, d in itertools.product(
            ("direct", "scanner_axis"),
            ("direct", "position_axis", "fastgs_conjugate", "position_conjugate"),
            ("wxyz", "xyzw"), ("sh", "raw_rgb"), ("sh", "rgb"), (deg, 1)):
        if src == "rgb" and d != deg:
            continue
        record.clear()
        model = sh_model if src == "sh" else rgb_model
        # the path's folder exists (the reference creates it otherwise); the
        # stand-in writes nothing
        R.export_trained_spz(Path(HERE) / "unused.spz", model, src, d, scale, rot, order, color)
        c = record[0]
        tag = f"{scale}.{rot}.{order}.{color}.{src}.{d}"
        cases.append(tag)
        for f in ("positions", "scales", "rotations", "alphas", "colors", "sh"):
            out[f"{tag}.{f}"] = np.asarray(getattr(c, f), np.float32)
        out[f"{tag}.sh_degree"] = np.int32(c.sh_degree)
    out["cases"] = np.array(cases)
    np.savez_compressed(os.path.join(HERE, "formats.npz"), **out)
    R.save_model_parameters_npz(Path(os.path.join(HERE, "checkpoint_sh.npz")), sh_model, "sh", 2,
                                deg, {"step": 1234, "note": "golden"})
    print(len(cases), "export cases")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else
         os.path.join(os.sep, "root", "reference", "scripts", "test"))
