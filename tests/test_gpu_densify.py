"""On-device densification statistics (gsplat_core.densify) against the
reference trainer's own ScannerDefaultStrategyRuntime outputs
(tests/golden/densify.npz) and the CPU oracle: the accumulated statistics
bit for bit; the masks exactly, except where a scale or opacity lies within
a few ulp of its threshold (expf against numpy's exp), which the test
counts and requires to be rare."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from _util import assert_exact, to_np

pytestmark = pytest.mark.gpu


def T(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def _cfg(d):
    from gsplat_core.densify import DensifyConfig
    return DensifyConfig(prune_opa=float(d["prune_opa"]), grow_grad2d=float(d["grow_grad2d"]),
                         grow_scale3d=float(d["grow_scale3d"]), grow_scale2d=float(d["grow_scale2d"]),
                         prune_scale3d=float(d["prune_scale3d"]),
                         prune_scale2d=float(d["prune_scale2d"]),
                         refine_scale2d_stop_iter=int(d["refine_scale2d_stop_iter"]),
                         reset_every=int(d["reset_every"]), scene_scale=float(d["scene_scale"]))


def _near(x, thr, ulps=4):
    x = np.asarray(x, np.float32)
    return np.abs(x - np.float32(thr)) <= ulps * np.spacing(np.abs(np.float32(thr)))


def test_densify_statistics_and_masks_match_reference(golden, cuda):
    from gsplat_core.densify import DensifyStats
    d = golden("densify")
    n, C, W, H = int(d["N"]), int(d["C"]), int(d["W"]), int(d["H"])
    st = DensifyStats(n, _cfg(d))
    for t in range(d["v_means2d"].shape[0]):
        st.update_state(T(d["v_means2d"][t]), T(d["radii_in"][t]), W, H, C)
    assert_exact(to_np(st.grad2d), d["grad2d"], "grad2d")
    assert_exact(to_np(st.count), d["count"], "count")
    assert_exact(to_np(st.radii), d["radii"], "radii")
    step = int(d["step"])
    m = st.masks(step, T(d["log_scales"]), T(d["opacity_logits"]), n, grow=True, prune=False)
    max_scale = np.exp(d["log_scales"]).max(axis=-1)
    edge = _near(max_scale, float(d["grow_scale3d"]) * float(d["scene_scale"]))
    clone_ref = np.zeros(n, bool)
    clone_ref[d["clone_selected"]] = True
    bad = (to_np(m["clone"]) != clone_ref) & ~edge
    assert not bad.any(), np.nonzero(bad)[0][:10]
    bad = (to_np(m["split"]) != d["split_mask"][:n]) & ~edge
    assert not bad.any(), np.nonzero(bad)[0][:10]
    assert edge.mean() < 1e-3
    assert m["n_clone"] == int(to_np(m["clone"]).sum()) and m["n_split"] == int(to_np(m["split"]).sum())
    # the prune mask on the state after the reference's clone and split
    st.radii = T(d["prune_radii"])
    p = st.masks(step, T(d["prune_log_scales"]), T(d["prune_opacity_logits"]), grow=False,
                 prune=True)
    keep_ref = np.ones(len(d["prune_opacity_logits"]), bool)
    keep_ref[:] = False
    keep_ref[d["prune_keep"]] = True
    o = 1.0 / (1.0 + np.exp(-d["prune_opacity_logits"]))
    edge = (_near(o, float(d["prune_opa"])) |
            _near(np.exp(d["prune_log_scales"]).max(axis=-1),
                  float(d["prune_scale3d"]) * float(d["scene_scale"])))
    bad = (~to_np(p["prune"]) != keep_ref) & ~edge
    assert not bad.any(), np.nonzero(bad)[0][:10]
    if not edge.any():
        assert p["prune_breakdown"] == d["prune_breakdown"].tolist()


def test_densify_state_bookkeeping_follows_topology(cuda):
    """apply_duplicate / apply_split / apply_keep reorder the statistics the
    way the reference's _apply_*_to_state do (:467-472, :497-502, :586-592)."""
    from gsplat_core.densify import DensifyConfig, DensifyStats
    st = DensifyStats(5, DensifyConfig(refine_scale2d_stop_iter=10))
    st.grad2d.copy_(torch.arange(5, dtype=torch.float32))
    st.count.copy_(torch.arange(5, dtype=torch.float32) + 10)
    st.radii.copy_(torch.arange(5, dtype=torch.float32) + 20)
    st.apply_duplicate(torch.tensor([1, 3], device="cuda"))
    assert to_np(st.grad2d).tolist() == [0, 1, 2, 3, 4, 1, 3]
    split = torch.tensor([False, True, False, False, True, False, False], device="cuda")
    st.apply_split(split)
    assert to_np(st.grad2d).tolist() == [0, 2, 3, 1, 3, 1, 4, 1, 4]
    st.apply_keep(torch.tensor([0, 2, 8], device="cuda"))
    assert to_np(st.count).tolist() == [10, 13, 14]
    assert to_np(st.radii).tolist() == [20, 23, 24]
