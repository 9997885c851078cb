"""Host-side validation of the drop-in functions: the reference's error
messages (gsplat_core/*.cpp front-ends, binding.cpp) raised as
RuntimeError before any device work -- runs on CPU tensors."""
from __future__ import annotations

import numpy as np
import pytest
import torch


def test_missing_required_key(gs):
    with pytest.raises(RuntimeError, match="missing input: means"):
        gs.projection_ewa_3dgs_fused_forward({"viewmats": np.eye(4)}, 8, 8)


def test_projection_shape_errors(gs):
    v = torch.eye(4)[None, None]
    K = torch.eye(3)[None, None]
    with pytest.raises(RuntimeError, match=r"means must have shape \[..., N, 3\]"):
        gs.projection_ewa_3dgs_fused_forward({"means": torch.zeros(1, 4, 2), "viewmats": v, "Ks": K}, 8, 8)
    with pytest.raises(RuntimeError, match="covars or quats"):
        gs.projection_ewa_3dgs_fused_forward({"means": torch.zeros(1, 4, 3), "viewmats": v, "Ks": K}, 8, 8)
    with pytest.raises(RuntimeError, match="viewspace_points"):
        gs.projection_ewa_3dgs_fused_forward(
            {"means": torch.zeros(1, 4, 3), "viewmats": v, "Ks": K, "covars": torch.zeros(1, 4, 6),
             "viewspace_points": torch.zeros(1, 1, 3, 2)}, 8, 8)


def test_intersect_unsupported_paths(gs):
    base = {"means2d": torch.zeros(1, 3, 2), "radii": torch.zeros(1, 3, 2, dtype=torch.int32),
            "depths": torch.zeros(1, 3)}
    with pytest.raises(RuntimeError, match="packed path"):
        gs.intersect_tile_forward(dict(base, image_ids=torch.zeros(3, dtype=torch.int64)), 1, 16, 4, 4)
    with pytest.raises(RuntimeError, match="segmented sort"):
        gs.intersect_tile_forward(base, 1, 16, 4, 4, segmented=True)
    with pytest.raises(RuntimeError, match="AccuTile"):
        gs.intersect_tile_forward(dict(base, conics=torch.zeros(1, 3, 3)), 1, 16, 4, 4)
    with pytest.raises(RuntimeError, match="int32 radii"):
        gs.intersect_tile_forward(dict(base, radii=torch.zeros(1, 3, 2)), 1, 16, 4, 4)


def test_rasterize_and_sh_errors(gs):
    with pytest.raises(RuntimeError, match="packed path"):
        gs.rasterize_to_pixels_3dgs_forward(
            {"means2d": torch.zeros(3, 2), "conics": torch.zeros(3, 3), "colors": torch.zeros(3, 3),
             "opacities": torch.zeros(3), "tile_offsets": torch.zeros(1, 1, 1, dtype=torch.int32),
             "flatten_ids": torch.zeros(0, dtype=torch.int32)}, 16, 16, 16)
    with pytest.raises(RuntimeError, match="degree 0..4"):
        gs.spherical_harmonics_forward(5, {"dirs": torch.zeros(2, 3), "coeffs": torch.zeros(2, 36, 3)})
    with pytest.raises(RuntimeError, match="fewer SH bases"):
        gs.spherical_harmonics_forward(3, {"dirs": torch.zeros(2, 3), "coeffs": torch.zeros(2, 9, 3)})
    with pytest.raises(RuntimeError, match="same shape as dirs"):
        gs.spherical_harmonics_backward(1, {"dirs": torch.zeros(2, 3), "coeffs": torch.zeros(2, 4, 3)},
                                        {"v_colors": torch.zeros(3, 3)})


def test_quat_scale_errors(gs):
    with pytest.raises(RuntimeError, match=r"quats must have shape \[..., 4\]"):
        gs.quat_scale_to_covar_preci_forward({"quats": torch.zeros(2, 3), "scales": torch.zeros(2, 3)})
    with pytest.raises(RuntimeError, match="prefix dimensions"):
        gs.quat_scale_to_covar_preci_forward({"quats": torch.zeros(2, 4), "scales": torch.zeros(3, 3)})
    with pytest.raises(RuntimeError, match="v_covars shape"):
        gs.quat_scale_to_covar_preci_backward({"quats": torch.zeros(2, 4), "scales": torch.zeros(2, 3)},
                                              {"v_covars": torch.zeros(2, 3, 3)}, True)


def test_dummies(gs):
    assert gs.dummy_add(20, 22) == 42
    out = gs.dummy_array_add({"a": torch.tensor([1.0, 2.0, 3.0]), "b": torch.tensor([4.0, 5.0, 6.0])})
    assert out.tolist() == [5.0, 7.0, 9.0]
