"""The whole training step on the GPU (gsplat_core.pipeline.TrainingStep)
against the oracle's composition of the same operators, plus size-
independent properties at the full benchmark size."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from _util import assert_exact, assert_grad_close, to_np

pytestmark = pytest.mark.gpu


def T(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def oracle_step(oracle, sc, idx, vrc, vra):
    means, quats, scales = sc.means[idx], sc.quats[idx], sc.scales[idx]
    opac, coeffs = sc.opacities[idx], sc.coeffs[idx]
    W, H, ts, tw, th = sc.width, sc.height, sc.tile_size, sc.tile_width, sc.tile_height
    C = sc.cameras
    p = oracle.proj_fwd(means[None], sc.viewmats[None], sc.Ks[None], W, H, quats=quats[None],
                        scales=scales[None])
    vis = (p["radii"][0, ..., 0] > 0) & (p["radii"][0, ..., 1] > 0)
    colors = oracle.sh_glue_fwd(sc.sh_degree, means, sc.viewmats, coeffs, vis)
    m2 = p["means2d"].reshape(C, -1, 2)
    it = oracle.isect_tile(m2, p["radii"].reshape(C, -1, 2), p["depths"].reshape(C, -1), C, ts, tw, th)
    offs = oracle.isect_offset(it["isect_ids"], C, tw, th)
    op = np.broadcast_to(opac, (C, opac.size)).copy()
    bg = np.zeros((C, 3), np.float32)
    kw = dict(means2d=m2, conics=p["conics"].reshape(C, -1, 3), colors=colors, opacities=op,
              tile_offsets=offs, flatten_ids=it["flatten_ids"], width=W, height=H, tile_size=ts,
              backgrounds=bg)
    rf = oracle.raster_fwd(**kw)
    near = rf["near_threshold"]
    vrc = vrc.copy()
    vra = vra.copy()
    vrc[near] = 0
    vra[near] = 0
    rb = oracle.raster_bwd(render_alphas=rf["render_alphas"], last_ids=rf["last_ids"],
                           v_render_colors=vrc, v_render_alphas=vra, **kw)
    pb = oracle.proj_bwd(means[None], sc.viewmats[None], sc.Ks[None], W, H, p["radii"], p["conics"],
                         rb["v_means2d"][None], np.zeros(p["depths"].shape, np.float32),
                         rb["v_conics"][None], quats=quats[None], scales=scales[None])
    gb = oracle.sh_glue_bwd(sc.sh_degree, means, sc.viewmats, coeffs, rb["v_colors"], vis)
    grads = {"v_means": pb["v_means"][0] + gb["v_means"], "v_quats": pb["v_quats"][0],
             "v_scales": pb["v_scales"][0], "v_opacities": rb["v_opacities"].sum(0),
             "v_coeffs": gb["v_coeffs"]}
    return rf, it, offs, grads, vrc, vra, near


@pytest.mark.parametrize("n,cams", [(30_000, 1), (20_000, 3)])
def test_training_step_matches_oracle(gs, oracle, cuda, n, cams):
    from gsplat_core import pipeline, synthetic as S
    sc = S.config3(seed=1, n=200_000)
    if cams > 1:
        views = S.orbit(cams, 4.0)
        sc.viewmats = views
        sc.Ks = np.repeat(sc.Ks[:1], cams, 0)
    # quarter resolution keeps the oracle quick
    sc.Ks = sc.Ks.copy()
    sc.Ks[:, :2, :] /= 4
    sc.width, sc.height = sc.width // 4, sc.height // 4
    rng = np.random.default_rng(0)
    idx = np.sort(rng.choice(sc.n, size=n, replace=False))
    vrc, vra = S.cotangents(3, cams, sc.height, sc.width)
    rf, it, offs, eg, vrc, vra, near = oracle_step(oracle, sc, idx, vrc, vra)
    # the reference's full lists (the tile-culled ones are pinned in test_gpu_tile_cull)
    step = pipeline.TrainingStep(n, 3, 16, cams, sc.width, sc.height, tile_cull=False)
    flat, m = step.run(T(sc.means[idx]), T(sc.quats[idx]), T(sc.scales[idx]),
                       T(sc.opacities[idx]), T(sc.coeffs[idx]), T(sc.viewmats), T(sc.Ks),
                       T(vrc), T(vra))
    torch.cuda.synchronize()
    step.check()   # no bounded on-device wait of the sort gave up
    assert m == it["isect_ids"].size
    assert_exact(step.sorted_ids[:m], it["isect_ids"], "sorted keys")
    assert_exact(step.sorted_flatten[:m], it["flatten_ids"], "sorted flatten ids")
    assert_exact(step.tile_offsets, offs, "tile offsets")
    ok = ~near
    assert_exact(to_np(step.last_ids)[ok], rf["last_ids"][ok], "last ids")
    for k, v in step.gradients().items():
        assert_grad_close(v, eg[k], k, atol_frac=1e-4)


def test_full_size_config3_properties(gs, oracle, cuda):
    """BASELINE config 3 at full size (1M Gaussians, SH3, 1297x840):
    intersection count equals the oracle's, keys are sorted, offsets are the
    bucket boundaries, outputs are finite and alphas in [0, 1]."""
    from gsplat_core import pipeline, synthetic as S
    sc = S.config3(seed=0)
    vrc, vra = S.cotangents(0, 1, sc.height, sc.width)
    step = pipeline.TrainingStep(sc.n, 3, 16, 1, sc.width, sc.height, tile_cull=False)
    args = [T(sc.means), T(sc.quats), T(sc.scales), T(sc.opacities), T(sc.coeffs),
            T(sc.viewmats), T(sc.Ks), T(vrc), T(vra)]
    flat, m = step.run(*args)
    torch.cuda.synchronize()
    step.check()
    p = oracle.proj_fwd(sc.means[None], sc.viewmats[None], sc.Ks[None], sc.width, sc.height,
                        quats=sc.quats[None], scales=sc.scales[None])
    assert_exact(step.radii[0], p["radii"][0, 0], "radii")
    tpg = np.zeros(sc.n, np.int32)
    oracle.lib.orc_isect_count(1, sc.n, p["means2d"].ctypes.data, p["radii"].ctypes.data,
                               16, sc.tile_width, sc.tile_height, tpg.ctypes.data)
    assert m == int(tpg.astype(np.int64).sum())
    ids = step.sorted_ids[:m]
    assert bool((ids[1:] >= ids[:-1]).all())
    hi = (ids >> 32).cpu().numpy()
    offs = to_np(step.tile_offsets).ravel()
    ntiles = sc.tile_width * sc.tile_height
    expect = np.searchsorted(hi, np.arange(ntiles), side="left")
    assert_exact(offs, expect, "offsets")
    ra = to_np(step.render_alphas)
    assert np.isfinite(ra).all() and ra.min() >= 0 and ra.max() <= 1
    g = to_np(flat)
    assert np.isfinite(g).all() and np.abs(g).max() > 0
    # The same step again gives the same intersections and the same image.
    last0 = step.last_ids.clone()
    flat2, m2 = step.run(*args)
    torch.cuda.synchronize()
    assert m2 == m
    assert torch.equal(last0, step.last_ids)
    assert_grad_close(flat2, g, "repeat step", atol_frac=1e-5)



@pytest.mark.parametrize("tile_cull", [False, True])
def test_banded_passes_match_one_pass(gs, cuda, tile_cull):
    """Past max_isects_per_pass the step renders bands of tile rows, each
    with its own intersection pass: the same image bit for bit, and the
    same gradients up to the order of the atomic additions."""
    from gsplat_core import pipeline, synthetic as S
    sc = S.config3(seed=2, n=200_000)
    views = S.orbit(2, 4.0)
    Ks = np.repeat(sc.Ks[:1], 2, 0).copy()
    Ks[:, :2, :] /= 4
    W, H = sc.width // 4, sc.height // 4
    idx = np.sort(np.random.default_rng(1).choice(sc.n, size=30_000, replace=False))
    vrc, vra = S.cotangents(8, 2, H, W)
    args = [T(sc.means[idx]), T(sc.quats[idx]), T(sc.scales[idx]), T(sc.opacities[idx]),
            T(sc.coeffs[idx]), T(views), T(Ks), T(vrc), T(vra)]
    one = pipeline.TrainingStep(idx.size, 3, 16, 2, W, H, tile_cull=tile_cull)
    flat1, m1 = one.run(*args)
    flat1 = flat1.clone()
    banded = pipeline.TrainingStep(idx.size, 3, 16, 2, W, H, max_isects_per_pass=m1 // 3,
                                   tile_cull=tile_cull)
    flat2, m2 = banded.run(*args)
    torch.cuda.synchronize()
    banded.check()
    assert one.bands == 1 and banded.bands > 2
    assert m2 == m1
    assert torch.equal(one.render_colors, banded.render_colors)
    assert torch.equal(one.render_alphas, banded.render_alphas)
    assert_grad_close(flat2, flat1, "banded vs one pass", atol_frac=1e-4)
