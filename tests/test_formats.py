"""On-disk formats (gsplat_core.formats) on the CPU: the oracle's SPZ
conversions against the reference's own export_trained_spz output, and the
npz parameter checkpoint against the file the reference's
save_model_parameters_npz wrote (tests/golden/make_formats_golden.py)."""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch

from oracle.formats import spz_attributes as oracle_spz

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
FIELDS = ("positions", "scales", "rotations", "alphas", "colors", "sh")


def _cases():
    g = np.load(os.path.join(GOLDEN, "formats.npz"))
    return g, [str(t) for t in g["cases"]]


def _inputs(g, src):
    q = g["quats"]
    q = q / np.maximum(np.sqrt(np.sum(q * q, axis=-1, keepdims=True)), np.float32(1e-8))
    col = 1.0 / (1.0 + np.exp(-g["color_logits"])) if src == "rgb" else g["features_dc"]
    return g["means"], q, g["log_scales"], g["opacity_logits"], col, g["features_rest"]


def test_oracle_matches_reference_export():
    g, cases = _cases()
    assert len(cases) == 96
    for tag in cases:
        scale, rot, order, color, src, d = tag.split(".")
        o = oracle_spz(*_inputs(g, src), scale, rot, order, color, src, int(d))
        for f in FIELDS:
            np.testing.assert_array_equal(np.asarray(o[f], np.float32).reshape(-1),
                                          g[f"{tag}.{f}"], err_msg=f"{tag} {f}")
        assert o["sh_degree"] == int(g[f"{tag}.sh_degree"])


def test_checkpoint_npz_matches_reference_writer(tmp_path):
    from gsplat_core import formats
    ref = np.load(os.path.join(GOLDEN, "checkpoint_sh.npz"))
    g, _ = _cases()
    T = torch.from_numpy
    path = tmp_path / "ckpt" / "params.npz"
    formats.save_checkpoint_npz(path, T(g["means"]), T(g["quats"]), T(g["log_scales"]),
                                T(g["opacity_logits"]), features_dc=T(g["features_dc"]),
                                features_rest=T(g["features_rest"]), active_sh_degree=2,
                                max_sh_degree=3, summary={"step": 1234, "note": "golden"})
    ours = np.load(path)
    assert sorted(ours.files) == sorted(ref.files)
    for k in ref.files:
        assert ours[k].dtype == ref[k].dtype and ours[k].shape == ref[k].shape, k
        np.testing.assert_array_equal(ours[k], ref[k], err_msg=k)
    back = formats.load_checkpoint_npz(path)
    assert back["color_mode"] == "sh" and back["active_sh_degree"] == 2
    assert back["summary"] == {"step": 1234, "note": "golden"}
    np.testing.assert_array_equal(back["features_rest"].numpy(), g["features_rest"])
    np.testing.assert_array_equal(back["quats_wxyz"].numpy(), ref["quats_wxyz"][0])


def test_rgb_checkpoint_round_trip(tmp_path):
    from gsplat_core import formats
    rng = np.random.default_rng(2)
    n = 33
    a = {k: torch.from_numpy(rng.normal(size=s).astype(np.float32)) for k, s in
         (("means", (n, 3)), ("quats", (n, 4)), ("log_scales", (n, 3)),
          ("opacity_logits", (n,)), ("color_logits", (n, 3)))}
    path = tmp_path / "rgb.npz"
    formats.save_checkpoint_npz(path, a["means"], a["quats"], a["log_scales"],
                                a["opacity_logits"], color_logits=a["color_logits"])
    d = np.load(path)
    assert str(d["color_mode"]) == "rgb" and d["color_logits"].shape == (1, 1, n, 3)
    back = formats.load_checkpoint_npz(path)
    for k in ("means", "log_scales", "opacity_logits", "color_logits"):
        assert torch.equal(back[k], a[k]), k


def test_spz_mode_errors():
    from gsplat_core import formats
    z = torch.zeros((1, 3))
    with pytest.raises(ValueError, match="Unsupported SPZ color mode"):
        formats.spz_attributes(z, torch.zeros((1, 4)), z, torch.zeros(1), features_dc=z,
                               color_mode="hsv")
    with pytest.raises(ValueError, match="features_dc"):
        formats.spz_attributes(z, torch.zeros((1, 4)), z, torch.zeros(1))
