"""Opacity-aware tile culling of the binned encode
(gs_isect_tile_encode_binned_culled, intersect_tile_culled_forward, the
training step's opt-in tile_cull).  The reference's intersect_tile_forward refuses
conics / opacities (gsplat_intersect.cpp:115-126), so there is no reference
list to match; the culled lists are pinned to the reference's full lists
instead:

* the culled list is the full (reference-identical) list with some
  (tile, Gaussian) pairs taken out, order kept, bit for bit, and its tile
  offsets are the bucket boundaries of its keys;
* every pair taken out stays below alpha 1/255 at all 256 pixel centres of
  its tile, evaluated in float64 (so the rasterizer skips it everywhere);
* rasterizing either list gives the same colours and alphas bit for bit,
  the same last composited Gaussian per pixel, and gradients equal up to
  the order of the atomic additions.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from _util import assert_exact, assert_grad_close, to_np

pytestmark = pytest.mark.gpu


def T(x, dev="cuda"):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


def _scene(n, cams, seed=0, scale=4):
    """A config-3 subset seen by `cams` orbit cameras at 1/scale resolution."""
    from gsplat_core import synthetic as S
    sc = S.config3(seed=seed, n=max(4 * n, 10))
    idx = np.sort(np.random.default_rng(seed + 1).choice(sc.n, size=n, replace=False))
    views = S.orbit(cams, 4.0) if cams > 1 else sc.viewmats
    Ks = np.repeat(sc.Ks[:1], cams, 0).copy()
    Ks[:, :2, :] /= scale
    return sc, idx, views, Ks, sc.width // scale, sc.height // scale


def _project(gs, sc, idx, views, Ks, W, H):
    inp = {"means": T(sc.means[idx][None]), "quats": T(sc.quats[idx][None]),
           "scales": T(sc.scales[idx][None]), "viewmats": T(views[None]), "Ks": T(Ks[None])}
    p = gs.projection_ewa_3dgs_fused_forward(inp, W, H)
    C, N = views.shape[0], idx.size
    opac = T(np.repeat(sc.opacities[idx][None], C, 0))
    return {"means2d": p["means2d"].view(C, N, 2), "radii": p["radii"].view(C, N, 2),
            "depths": p["depths"].view(C, N), "conics": p["conics"].view(C, N, 3),
            "opacities": opac}


def _max_alpha(m2, con, op, tiles, gids, tw, ts=16):
    """float64 max over the tile's pixel centres of o exp(-sigma)."""
    out = np.empty(gids.size)
    off = np.arange(ts) + 0.5
    for a in range(0, gids.size, 4096):
        g, t = gids[a:a + 4096], tiles[a:a + 4096]
        px = (t % tw)[:, None] * ts + off[None, :]          # [k, ts]
        py = (t // tw)[:, None] * ts + off[None, :]
        dx = m2[g, 0][:, None, None] - px[:, None, :]        # [k, 1, ts] (columns)
        dy = m2[g, 1][:, None, None] - py[:, :, None]        # [k, ts, 1] (rows)
        c0, c1, c2 = (con[g, i][:, None, None] for i in range(3))
        sig = 0.5 * (c0 * dx * dx + c2 * dy * dy) + c1 * dx * dy
        out[a:a + 4096] = op[g] * np.exp(-sig.reshape(g.size, -1).min(axis=1))
    return out


@pytest.mark.parametrize("cams", [1, 2])
def test_culled_lists_filter_the_full_lists(gs, cuda, cams):
    sc, idx, views, Ks, W, H = _scene(30_000, cams)
    ts, tw, th = 16, (W + 15) // 16, (H + 15) // 16
    f = _project(gs, sc, idx, views, Ks, W, H)
    full = gs.intersect_tile_forward({k: f[k] for k in ("means2d", "radii", "depths")}, cams,
                                     ts, tw, th)
    cul = gs.intersect_tile_culled_forward(f, cams, ts, tw, th)
    m, kept = full["isect_ids"].numel(), cul["isect_ids"].numel()
    assert 0 < kept < m, (kept, m)
    fid, ffl = to_np(full["isect_ids"]), to_np(full["flatten_ids"]).astype(np.int64)
    cid, cfl = to_np(cul["isect_ids"]), to_np(cul["flatten_ids"]).astype(np.int64)
    n_el = cams * idx.size
    fkey, ckey = (fid >> 32) * n_el + ffl, (cid >> 32) * n_el + cfl
    keep = np.isin(fkey, ckey)
    assert int(keep.sum()) == kept
    assert_exact(fid[keep], cid, "culled keys = full keys filtered")
    assert_exact(ffl[keep], cfl, "culled flatten ids = full flatten ids filtered")
    assert_exact(cul["tile_offsets"],
                 to_np(gs.intersect_offset_forward(cul["isect_ids"], cams, tw, th)),
                 "culled tile offsets")
    # every dropped pair is below 1/255 at every pixel centre of its tile
    tile_bits = int(tw * th).bit_length()
    drop = ~keep
    tiles = (fid[drop] >> 32) & ((1 << tile_bits) - 1)
    amax = _max_alpha(to_np(f["means2d"]).reshape(-1, 2).astype(np.float64),
                      to_np(f["conics"]).reshape(-1, 3).astype(np.float64),
                      to_np(f["opacities"]).reshape(-1).astype(np.float64), tiles, ffl[drop], tw)
    assert (amax < 1.0 / 255.0).all(), (amax.max(), int((amax >= 1.0 / 255.0).sum()))


def test_culled_render_and_gradients_match(gs, cuda):
    from gsplat_core import synthetic as S
    cams = 2
    sc, idx, views, Ks, W, H = _scene(30_000, cams, seed=3)
    ts, tw, th = 16, (W + 15) // 16, (H + 15) // 16
    f = _project(gs, sc, idx, views, Ks, W, H)
    full = gs.intersect_tile_forward({k: f[k] for k in ("means2d", "radii", "depths")}, cams,
                                     ts, tw, th)
    foff = gs.intersect_offset_forward(full["isect_ids"], cams, tw, th)
    cul = gs.intersect_tile_culled_forward(f, cams, ts, tw, th)
    rng = np.random.default_rng(5)
    colors = T(rng.uniform(0, 1, size=(cams, idx.size, 3)).astype(np.float32))
    bg = T(rng.uniform(0, 1, size=(cams, 3)).astype(np.float32))
    base = {"means2d": f["means2d"], "conics": f["conics"], "colors": colors,
            "opacities": f["opacities"], "backgrounds": bg}
    rin_f = dict(base, tile_offsets=foff, flatten_ids=full["flatten_ids"])
    rin_c = dict(base, tile_offsets=cul["tile_offsets"], flatten_ids=cul["flatten_ids"])
    rf = gs.rasterize_to_pixels_3dgs_forward(rin_f, W, H, ts)
    rc = gs.rasterize_to_pixels_3dgs_forward(rin_c, W, H, ts)
    assert torch.equal(rf["render_colors"], rc["render_colors"])
    assert torch.equal(rf["render_alphas"], rc["render_alphas"])
    hit = to_np(rf["render_alphas"])[..., 0] > 0
    gf = to_np(full["flatten_ids"])[to_np(rf["last_ids"])[hit]]
    gc = to_np(cul["flatten_ids"])[to_np(rc["last_ids"])[hit]]
    assert_exact(gc, gf, "last composited Gaussian per pixel")
    vrc, vra = S.cotangents(2, cams, H, W)
    cot = {"v_render_colors": T(vrc), "v_render_alphas": T(vra)}
    bf = gs.rasterize_to_pixels_3dgs_backward(rin_f, rf, cot, W, H, ts, absgrad=True)
    bc = gs.rasterize_to_pixels_3dgs_backward(rin_c, rc, cot, W, H, ts, absgrad=True)
    for k in ("v_means2d", "v_means2d_abs", "v_conics", "v_colors", "v_opacities",
              "v_backgrounds"):
        assert_grad_close(bc[k], bf[k], "culled vs full " + k, atol_frac=1e-5)


@pytest.mark.parametrize("full_size", [False, True])
def test_training_step_tile_cull(gs, cuda, full_size):
    """The training step with and without culling: the same renders bit for
    bit, gradients equal up to atomic order, fewer intersections walked;
    the culled keys sit sorted in the last places of the lists, with the
    tile offsets pointing at their buckets.  full_size: benchmark config 3
    (1M Gaussians, 1297x840)."""
    from gsplat_core import pipeline, synthetic as S
    if full_size:
        sc = S.config3(seed=0)
        idx, views, Ks, W, H, cams = np.arange(sc.n), sc.viewmats, sc.Ks, sc.width, sc.height, 1
    else:
        cams = 2
        sc, idx, views, Ks, W, H = _scene(40_000, cams, seed=4)
    vrc, vra = S.cotangents(1, cams, H, W)
    args = [T(sc.means[idx]), T(sc.quats[idx]), T(sc.scales[idx]), T(sc.opacities[idx]),
            T(sc.coeffs[idx]), T(views), T(Ks), T(vrc), T(vra)]
    ref = pipeline.TrainingStep(idx.size, 3, 16, cams, W, H, tile_cull=False)
    g0, m0 = ref.run(*args)
    g0 = g0.clone()
    step = pipeline.TrainingStep(idx.size, 3, 16, cams, W, H, tile_cull=True)
    assert step.tile_cull
    g1, m1 = step.run(*args)
    torch.cuda.synchronize()
    step.check()
    assert m1 == m0
    kept = step.kept_isects()
    assert 0 < kept < m1
    assert torch.equal(ref.render_colors, step.render_colors)
    assert torch.equal(ref.render_alphas, step.render_alphas)
    assert_grad_close(g1, g0, "culled vs full step", atol_frac=1e-4)
    gap = m1 - kept
    ids = step.sorted_ids[gap:m1]
    assert bool((ids[1:] >= ids[:-1]).all())
    tw, th = (W + 15) // 16, (H + 15) // 16
    tile_bits = int(tw * th).bit_length()
    hi = (ids >> 32).cpu().numpy()
    keys = (np.arange(cams)[:, None] << tile_bits) + np.arange(tw * th)[None, :]
    expect = gap + np.searchsorted(hi, keys.ravel(), side="left")
    assert_exact(to_np(step.tile_offsets).ravel(), expect, "culled step offsets")
