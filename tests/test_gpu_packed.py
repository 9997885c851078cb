"""Packed [nnz] layout (gsplat_core.packed) against the dense path, which
is pinned to the reference elsewhere.  The reference refuses packed inputs
(gsplat_intersect.cpp:115-118), so the packed results are pinned to the
dense ones: the rows are the dense outputs' visible entries bit for bit; the
sorted keys and tile offsets equal the dense ones bit for bit, with each
flatten id naming the row of the same (image, Gaussian); renders are
bit-identical and the per-row gradients equal the dense gradients at those
entries up to the order of the atomic additions."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from _util import assert_exact, assert_grad_close, to_np

pytestmark = pytest.mark.gpu


def T(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


@pytest.mark.parametrize("cams,comp", [(1, False), (3, True)])
def test_packed_path_matches_dense(gs, cuda, cams, comp):
    from gsplat_core import packed as P, synthetic as S
    sc = S.config3(seed=6, n=120_000)
    idx = np.sort(np.random.default_rng(7).choice(sc.n, size=40_000, replace=False))
    views = S.orbit(cams, 4.0) if cams > 1 else sc.viewmats
    Ks = np.repeat(sc.Ks[:1], cams, 0).copy()
    Ks[:, :2, :] /= 4
    W, H = sc.width // 4, sc.height // 4
    N = idx.size
    ts, tw, th = 16, (W + 15) // 16, (H + 15) // 16
    proj = gs.projection_ewa_3dgs_fused_forward(
        {"means": T(sc.means[idx][None]), "quats": T(sc.quats[idx][None]),
         "scales": T(sc.scales[idx][None]), "viewmats": T(views[None]), "Ks": T(Ks[None])},
        W, H, calc_compensations=comp)
    pk = P.pack_projection(proj)
    # rows: the visible dense entries, in (image, Gaussian) order
    r = to_np(proj["radii"]).reshape(cams * N, 2)
    vis = np.flatnonzero((r[:, 0] > 0) & (r[:, 1] > 0))
    assert 0 < vis.size < cams * N
    assert_exact(pk["image_ids"], (vis // N).astype(np.int32), "image ids")
    assert_exact(pk["gaussian_ids"], (vis % N).astype(np.int32), "gaussian ids")
    for k, w in (("radii", 2), ("means2d", 2), ("depths", 1), ("conics", 3)):
        assert_exact(pk[k], to_np(proj[k]).reshape(cams * N, w)[vis].reshape(pk[k].shape), k)
    if comp:
        assert_exact(pk["compensations"], to_np(proj["compensations"]).reshape(-1)[vis], "comps")
    # sorted lists: dense keys, flatten ids through the rows
    dense = gs.intersect_tile_forward({"means2d": proj["means2d"].view(cams, N, 2),
                                       "radii": proj["radii"].view(cams, N, 2),
                                       "depths": proj["depths"].view(cams, N)}, cams, ts, tw, th)
    doff = gs.intersect_offset_forward(dense["isect_ids"], cams, tw, th)
    it = P.intersect_tile_packed_forward(pk, cams, ts, tw, th)
    assert_exact(it["isect_ids"], dense["isect_ids"], "packed keys")
    assert_exact(vis[to_np(it["flatten_ids"])], to_np(dense["flatten_ids"]), "packed flatten ids")
    assert_exact(it["tile_offsets"], doff, "packed tile offsets")
    # rasterize: same images, gradients per row = dense gradients at the rows
    rng = np.random.default_rng(8)
    colors = rng.uniform(0, 1, size=(cams, N, 3)).astype(np.float32)
    opac = np.repeat(sc.opacities[idx][None], cams, 0)
    bg = T(rng.uniform(0, 1, size=(cams, 3)).astype(np.float32))
    rin = {"means2d": proj["means2d"].view(cams, N, 2), "conics": proj["conics"].view(cams, N, 3),
           "colors": T(colors), "opacities": T(opac), "backgrounds": bg,
           "tile_offsets": doff, "flatten_ids": dense["flatten_ids"]}
    pin = {"means2d": pk["means2d"], "conics": pk["conics"],
           "colors": T(colors.reshape(-1, 3)[vis]), "opacities": T(opac.reshape(-1)[vis]),
           "backgrounds": bg}
    rf = gs.rasterize_to_pixels_3dgs_forward(rin, W, H, ts)
    pf = P.rasterize_packed_forward(pin, it, cams, W, H, ts)
    assert torch.equal(rf["render_colors"], pf["render_colors"])
    assert torch.equal(rf["render_alphas"], pf["render_alphas"])
    hit = to_np(rf["render_alphas"])[..., 0] > 0
    assert_exact(vis[to_np(it["flatten_ids"])[to_np(pf["last_ids"])[hit]]],
                 to_np(dense["flatten_ids"])[to_np(rf["last_ids"])[hit]], "last ids")
    vrc, vra = S.cotangents(3, cams, H, W)
    cot = {"v_render_colors": T(vrc), "v_render_alphas": T(vra)}
    rb = gs.rasterize_to_pixels_3dgs_backward(rin, rf, cot, W, H, ts, absgrad=True)
    pb = P.rasterize_packed_backward(pin, it, pf, cot, cams, W, H, ts, absgrad=True)
    for k, w in (("v_means2d", 2), ("v_means2d_abs", 2), ("v_conics", 3), ("v_colors", 3),
                 ("v_opacities", 1)):
        e = to_np(rb[k]).reshape(cams * N, w)[vis].reshape(pb[k].shape)
        assert_grad_close(pb[k], e, "packed " + k, atol_frac=1e-5)
    assert_grad_close(pb["v_backgrounds"], rb["v_backgrounds"], "packed v_backgrounds")
    # and back to the dense layout for the projection backward
    back = P.unpack_rows(pb["v_means2d"], pk, cams, N)
    np.testing.assert_array_equal(to_np(back).reshape(-1, 2)[np.setdiff1d(
        np.arange(cams * N), vis)], 0.0)
    assert_grad_close(back, rb["v_means2d"].view(cams, N, 2), "unpacked v_means2d",
                      atol_frac=1e-5)


def test_packed_image_id_range_checked(gs, cuda):
    from gsplat_core import packed as P
    pk = {"image_ids": T(np.array([0, 2], np.int32)), "means2d": T(np.zeros((2, 2), np.float32)),
          "radii": T(np.ones((2, 2), np.int32)), "depths": T(np.ones(2, np.float32))}
    with pytest.raises(RuntimeError, match="image ids outside"):
        P.intersect_tile_packed_forward(pk, 2, 16, 4, 4)
