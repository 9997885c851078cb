"""The whole training step on the GPU (gsplat_core.pipeline.TrainingStep)
against the oracle's composition of the same operators, element by
element: at reduced sizes, at benchmark config 3's full size, with config
4's 32 cameras at 1920x1080, and with config 5's heavy overdraw in bands of
tile rows.  Integer outputs (radii, sorted keys, flatten ids, tile offsets,
last ids) are compared bit for bit on every entry, renders within 1e-5 abs
/ 1e-4 rel, gradients within 1e-3 rel (the atomic order differs)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from _util import assert_exact, assert_fwd_close, assert_grad_close, to_np

pytestmark = pytest.mark.gpu


def T(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def oracle_step(oracle, sc, idx, vrc, vra, noise=False):
    """The reference trainer's step (scanner_points_training_utils.py:
    2076-2119) composed from the oracle's operators.  With noise=True the
    backward runs a second time with another summation order (another
    thread count of the oracle's rasterizer) and "noise" holds the spread
    of each gradient entry between the two."""
    means, quats, scales = sc.means[idx], sc.quats[idx], sc.scales[idx]
    opac, coeffs = sc.opacities[idx], sc.coeffs[idx]
    W, H, ts, tw, th = sc.width, sc.height, sc.tile_size, sc.tile_width, sc.tile_height
    C = sc.viewmats.shape[0]
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

    def backward(threads):
        rb = oracle.raster_bwd(render_alphas=rf["render_alphas"], last_ids=rf["last_ids"],
                               v_render_colors=vrc, v_render_alphas=vra, threads=threads, **kw)
        pb = oracle.proj_bwd(means[None], sc.viewmats[None], sc.Ks[None], W, H, p["radii"],
                             p["conics"], rb["v_means2d"][None],
                             np.zeros(p["depths"].shape, np.float32), rb["v_conics"][None],
                             quats=quats[None], scales=scales[None])
        gb = oracle.sh_glue_bwd(sc.sh_degree, means, sc.viewmats, coeffs, rb["v_colors"], vis)
        return {"v_means": pb["v_means"][0] + gb["v_means"], "v_quats": pb["v_quats"][0],
                "v_scales": pb["v_scales"][0], "v_opacities": rb["v_opacities"].sum(0),
                "v_coeffs": gb["v_coeffs"]}

    from oracle.oracle import raster_threads
    t = raster_threads()
    grads = backward(t)
    out = dict(proj=p, rf=rf, it=it, offs=offs, grads=grads)
    if noise:
        other = backward(t // 2 + 1 if t > 2 else t + 1)
        out["noise"] = {k: np.abs(grads[k] - other[k]) for k in grads}
    return out


def run_step(sc, idx, vrc, vra, **kw):
    from gsplat_core import pipeline
    C = sc.viewmats.shape[0]
    step = pipeline.TrainingStep(idx.size, 3, 16, C, sc.width, sc.height, tile_cull=False, **kw)
    args = [T(sc.means[idx]), T(sc.quats[idx]), T(sc.scales[idx]), T(sc.opacities[idx]),
            T(sc.coeffs[idx]), T(sc.viewmats), T(sc.Ks), T(vrc), T(vra)]
    flat, m = step.run(*args)
    torch.cuda.synchronize()
    step.check()   # no bounded on-device wait of the sort gave up
    return step, args, flat, m


def compare_step(step, m, e, lists=True):
    it = e["it"]
    assert_exact(step.radii, e["proj"]["radii"][0], "radii")
    if lists:
        assert m == it["isect_ids"].size
        assert_exact(step.sorted_ids[:m], it["isect_ids"], "sorted keys")
        assert_exact(step.sorted_flatten[:m], it["flatten_ids"], "sorted flatten ids")
        assert_exact(step.tile_offsets, e["offs"], "tile offsets")
        assert_exact(step.last_ids, e["rf"]["last_ids"], "last ids")
    assert_fwd_close(step.render_colors, e["rf"]["render_colors"], "render colors")
    assert_fwd_close(step.render_alphas, e["rf"]["render_alphas"], "render alphas")
    for k, v in step.gradients().items():
        assert_grad_close(v, e["grads"][k], k, atol_frac=1e-4,
                          noise=e.get("noise", {}).get(k))


@pytest.mark.parametrize("n,cams", [(30_000, 1), (20_000, 3)])
def test_training_step_matches_oracle(gs, oracle, cuda, n, cams):
    from gsplat_core import synthetic as S
    sc = S.config3(seed=1, n=200_000)
    if cams > 1:
        sc.viewmats = S.orbit(cams, 4.0)
        sc.Ks = np.repeat(sc.Ks[:1], cams, 0)
    # quarter resolution keeps the oracle quick
    sc.Ks = sc.Ks.copy()
    sc.Ks[:, :2, :] /= 4
    sc.width, sc.height = sc.width // 4, sc.height // 4
    idx = np.sort(np.random.default_rng(0).choice(sc.n, size=n, replace=False))
    vrc, vra = S.cotangents(3, cams, sc.height, sc.width)
    e = oracle_step(oracle, sc, idx, vrc, vra)
    step, _, _, m = run_step(sc, idx, vrc, vra)
    compare_step(step, m, e)


def test_full_size_config3_matches_oracle(gs, oracle, cuda):
    """benchmark config 3 at full size (1M Gaussians, SH3, 1297x840, 6.9M
    intersections), every output element against the oracle; then the same
    step again gives the same lists and image bit for bit."""
    from gsplat_core import synthetic as S
    sc = S.config3(seed=0)
    idx = np.arange(sc.n)
    vrc, vra = S.cotangents(0, 1, sc.height, sc.width)
    e = oracle_step(oracle, sc, idx, vrc, vra)
    step, args, flat, m = run_step(sc, idx, vrc, vra)
    assert m > 6_000_000
    compare_step(step, m, e)
    last0, rc0 = step.last_ids.clone(), step.render_colors.clone()
    g0 = to_np(flat).copy()
    flat2, m2 = step.run(*args)
    torch.cuda.synchronize()
    assert m2 == m
    assert torch.equal(last0, step.last_ids) and torch.equal(rc0, step.render_colors)
    assert_grad_close(flat2, g0, "repeat step", atol_frac=1e-5)


def test_config4_cameras_match_oracle(gs, oracle, cuda):
    """benchmark config 4's batch (32 cameras at 1920x1080 on the 5 m orbit)
    over 100k Gaussians drawn from its 3M-Gaussian scene: every camera's
    lists, offsets, last ids and render, and the gradients summed over the
    32 cameras."""
    from gsplat_core import synthetic as S
    sc = S.config4(seed=0)
    idx = np.sort(np.random.default_rng(4).choice(sc.n, size=100_000, replace=False))
    vrc, vra = S.cotangents(4, sc.viewmats.shape[0], sc.height, sc.width)
    # 32 cameras' sums cancel heavily on some entries: allow for the spread
    # that another summation order gives the oracle itself
    e = oracle_step(oracle, sc, idx, vrc, vra, noise=True)
    step, _, _, m = run_step(sc, idx, vrc, vra)
    compare_step(step, m, e)


def test_config5_banded_matches_oracle(gs, oracle, cuda):
    """benchmark config 5's overdraw (log-scales U[-3,-1], one 3840x2160
    camera on the 3 m orbit) over 40k Gaussians of its 6M-Gaussian scene,
    rendered in bands of tile rows as the full config must be: each band's
    last ids are its own list's indices, i.e. the one-pass index minus the
    intersections of the rows above; renders and gradients as one pass."""
    from gsplat_core import synthetic as S
    sc = S.config5(seed=0)
    sc.viewmats, sc.Ks = sc.viewmats[:1].copy(), sc.Ks[:1].copy()
    idx = np.sort(np.random.default_rng(5).choice(sc.n, size=40_000, replace=False))
    vrc, vra = S.cotangents(5, 1, sc.height, sc.width)
    e = oracle_step(oracle, sc, idx, vrc, vra, noise=True)
    M = e["it"]["isect_ids"].size
    step, _, _, m = run_step(sc, idx, vrc, vra, max_isects_per_pass=M // 4)
    assert step.bands >= 3 and m == M
    compare_step(step, m, e, lists=False)
    # band-local last ids: subtract the first intersection of the pixel's band
    rows = max(1, int(sc.tile_height * step.max_isects_per_pass // (2 * M)))
    band_row0 = (np.arange(sc.tile_height) // rows) * rows
    base = e["offs"][0][band_row0, 0]                       # per tile row
    base_px = np.repeat(base, 16)[:sc.height][:, None]      # per pixel row
    ol, oa = e["rf"]["last_ids"][0], e["rf"]["render_alphas"][0, ..., 0]
    expect = np.where(oa == 0, 0, ol - base_px).astype(np.int32)
    assert_exact(to_np(step.last_ids)[0], expect, "band-local last ids")


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
