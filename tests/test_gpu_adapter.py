"""The C++ integration path on the GPU: the reference's own operator
front-ends (gsplat_core/*.cpp, compiled in the shim's device mode) with
every Primitive evaluated by the product's eval_gpu adapter
(gsplat-mlx_b200/adapter/gsplat_b200_eval_gpu.cpp), which calls the C ABI.

Checked element by element against the product's Python operators, which
launch the same kernels (integers and per-element floats bit-exact,
gradients summed with atomics within the summation-order tolerance), and
against the reference's eval_cpu (``Reference``) where the two paths share
their semantics (integers exact, floats within the parity tolerances)."""
from __future__ import annotations

import numpy as np
import pytest

from _util import assert_exact, assert_fwd_close, assert_grad_close, to_np

pytestmark = pytest.mark.gpu


def T(x, dev="cuda"):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


@pytest.fixture(scope="module")
def dev(cuda):
    from oracle.oracle import ReferenceOnDevice
    if not ReferenceOnDevice.available():
        pytest.skip("adapter build absent or built against another gsplat_b200.h "
                    "(make -C oracle ref_cuda REF=<reference tree>)")
    return ReferenceOnDevice()


@pytest.fixture(scope="module")
def ref():
    from oracle.oracle import Reference
    if not Reference.available():
        pytest.skip("reference eval_cpu build absent (make -C oracle ref)")
    return Reference()


@pytest.mark.parametrize("triu", [True, False])
def test_adapter_quat_scale(gs, dev, ref, triu):
    rng = np.random.default_rng(41)
    n = 5003
    q = rng.normal(size=(n, 4)).astype(np.float32)
    s = np.exp(rng.uniform(-3, 1, size=(n, 3))).astype(np.float32)
    a = dev.qs2c_fwd(q, s, True, True, triu)
    g = gs.quat_scale_to_covar_preci_forward({"quats": T(q), "scales": T(s)}, True, True, triu)
    e = ref.qs2c_fwd(q, s, True, True, triu)
    for k in ("covars", "precis"):
        assert_exact(a[k], to_np(g[k]), "adapter " + k)
        assert_fwd_close(a[k], e[k], "adapter vs eval_cpu " + k,
                         atol=1e-5 * max(1.0, np.abs(e[k]).max()))
    shape = (n, 6) if triu else (n, 3, 3)
    vc = rng.normal(size=shape).astype(np.float32)
    vp = rng.normal(size=shape).astype(np.float32)
    ab = dev.qs2c_bwd(q, s, vc, vp, triu)
    gb = gs.quat_scale_to_covar_preci_backward({"quats": T(q), "scales": T(s)},
                                               {"v_covars": T(vc), "v_precis": T(vp)}, triu)
    eb = ref.qs2c_bwd(q, s, vc, vp, triu)
    for k in ("v_quats", "v_scales"):
        assert_exact(ab[k], to_np(gb[k]), "adapter " + k)
        assert_grad_close(ab[k], eb[k], "adapter vs eval_cpu " + k)
    # only one cotangent given: the other is absent, not zero-filled input
    ab1 = dev.qs2c_bwd(q, s, vc, None, triu)
    gb1 = gs.quat_scale_to_covar_preci_backward({"quats": T(q), "scales": T(s)},
                                                {"v_covars": T(vc)}, triu)
    for k in ("v_quats", "v_scales"):
        assert_exact(ab1[k], to_np(gb1[k]), "adapter (covars only) " + k)


def _scene(n, seed=0):
    from gsplat_core import synthetic as S
    sc = S.config1(seed=seed)
    idx = np.sort(np.random.default_rng(seed + 1).choice(sc.n, size=min(n, sc.n), replace=False))
    return sc, idx


@pytest.mark.parametrize("comp", [False, True])
def test_adapter_projection(gs, dev, comp):
    sc, idx = _scene(8000)
    means, quats, scales = sc.means[idx][None], sc.quats[idx][None], sc.scales[idx][None]
    opac = sc.opacities[idx][None]
    W, H = sc.width, sc.height
    view, Ks = sc.viewmats[None], sc.Ks[None]
    a = dev.proj_fwd(means, view, Ks, W, H, quats=quats, scales=scales, opacities=opac,
                     calc_compensations=comp)
    g = gs.projection_ewa_3dgs_fused_forward(
        {"means": T(means), "quats": T(quats), "scales": T(scales), "opacities": T(opac),
         "viewmats": T(view), "Ks": T(Ks)}, W, H, calc_compensations=comp)
    for k in ("means2d", "depths", "conics", "radii"):
        assert_exact(a[k], to_np(g[k]), "adapter " + k)
    if comp:
        assert_exact(a["compensations"], to_np(g["compensations"]), "adapter compensations")
    else:
        assert a["compensations"].shape == (0,)
    rng = np.random.default_rng(7)
    shape = a["depths"].shape
    vm2 = rng.normal(size=shape + (2,)).astype(np.float32)
    vd = rng.normal(size=shape).astype(np.float32)
    vcon = rng.normal(size=shape + (3,)).astype(np.float32)
    vcomp = rng.normal(size=shape).astype(np.float32) if comp else None
    ab = dev.proj_bwd(means, view, Ks, W, H, a["radii"], a["conics"], vm2, vd, vcon,
                      quats=quats, scales=scales,
                      compensations=a["compensations"] if comp else None,
                      v_compensations=vcomp, viewmats_requires_grad=True)
    fo = {"radii": g["radii"], "conics": g["conics"]}
    cot = {"v_means2d": T(vm2), "v_depths": T(vd), "v_conics": T(vcon)}
    if comp:
        fo["compensations"] = g["compensations"]
        cot["v_compensations"] = T(vcomp)
    gb = gs.projection_ewa_3dgs_fused_backward(
        {"means": T(means), "quats": T(quats), "scales": T(scales), "viewmats": T(view),
         "Ks": T(Ks)}, fo, cot, W, H, viewmats_requires_grad=True)
    for k in ("v_means", "v_quats", "v_scales"):
        assert_exact(ab[k], to_np(gb[k]), "adapter " + k)
    assert_grad_close(ab["v_viewmats"], to_np(gb["v_viewmats"]), "adapter v_viewmats",
                      atol_frac=1e-4)


@pytest.mark.parametrize("deg,masked", [(0, False), (1, True), (3, False), (4, True)])
def test_adapter_spherical_harmonics(gs, dev, ref, deg, masked):
    rng = np.random.default_rng(50 + deg)
    n, K = 4001, (deg + 1) ** 2
    dirs = rng.normal(size=(n, 3)).astype(np.float32)
    coeffs = rng.normal(size=(n, K, 3)).astype(np.float32)
    masks = rng.uniform(size=n) < 0.7 if masked else None
    a = dev.sh_fwd(deg, dirs, coeffs, masks)
    inp = {"dirs": T(dirs), "coeffs": T(coeffs)}
    if masked:
        inp["masks"] = T(masks)
    g = gs.spherical_harmonics_forward(deg, inp)
    assert_exact(a, to_np(g["colors"] if isinstance(g, dict) else g), "adapter sh colors")
    assert_fwd_close(a, ref.sh_fwd(deg, dirs, coeffs, masks), "adapter vs eval_cpu colors")
    vcol = rng.normal(size=(n, 3)).astype(np.float32)
    ab = dev.sh_bwd(deg, dirs, coeffs, vcol, masks, compute_v_dirs=True)
    gb = gs.spherical_harmonics_backward(deg, inp, {"v_colors": T(vcol)}, compute_v_dirs=True)
    eb = ref.sh_bwd(deg, dirs, coeffs, vcol, masks, compute_v_dirs=True)
    for k in ("v_coeffs", "v_dirs"):
        assert_exact(ab[k], to_np(gb[k]), "adapter " + k)
        assert_grad_close(ab[k], eb[k], "adapter vs eval_cpu " + k)
    nd = dev.sh_bwd(deg, dirs, coeffs, vcol, masks, compute_v_dirs=False)
    assert "v_dirs" not in nd
    assert_exact(nd["v_coeffs"], ab["v_coeffs"], "adapter v_coeffs without v_dirs")


def _projected(gs, n=20000, seed=0):
    sc, idx = _scene(n, seed)
    g = gs.projection_ewa_3dgs_fused_forward(
        {"means": T(sc.means[idx][None]), "quats": T(sc.quats[idx][None]),
         "scales": T(sc.scales[idx][None]), "viewmats": T(sc.viewmats[None]),
         "Ks": T(sc.Ks[None])}, sc.width, sc.height)
    return sc, idx, {k: to_np(v) for k, v in g.items()}


def test_adapter_intersect_and_offsets(gs, dev, ref):
    sc, _, p = _projected(gs)
    m2 = p["means2d"].reshape(1, -1, 2)
    rad = p["radii"].reshape(1, -1, 2)
    dep = p["depths"].reshape(1, -1)
    tw, th, ts = sc.tile_width, sc.tile_height, sc.tile_size
    for sort in (False, True):
        a = dev.isect_tile(m2, rad, dep, 1, ts, tw, th, sort=sort)
        e = ref.isect_tile(m2, rad, dep, 1, ts, tw, th, sort=sort)
        g = gs.intersect_tile_forward({"means2d": T(m2), "radii": T(rad), "depths": T(dep)}, 1,
                                      ts, tw, th, sort=sort)
        for k in ("tiles_per_gauss", "isect_ids", "flatten_ids"):
            assert_exact(a[k], e[k], f"adapter vs eval_cpu {k} (sort={sort})")
            assert_exact(a[k], to_np(g[k]), f"adapter vs product {k} (sort={sort})")
    o = dev.isect_offset(a["isect_ids"], 1, tw, th)
    assert_exact(o, ref.isect_offset(e["isect_ids"], 1, tw, th), "adapter offsets")
    # two images, and an image with nothing on it
    m2b = np.concatenate([m2, m2], 0)
    radb = np.concatenate([rad, np.zeros_like(rad)], 0)
    depb = np.concatenate([dep, dep], 0)
    a2 = dev.isect_tile(m2b, radb, depb, 2, ts, tw, th)
    e2 = ref.isect_tile(m2b, radb, depb, 2, ts, tw, th)
    for k in ("tiles_per_gauss", "isect_ids", "flatten_ids"):
        assert_exact(a2[k], e2[k], "adapter two images " + k)
    assert_exact(dev.isect_offset(a2["isect_ids"], 2, tw, th),
                 ref.isect_offset(e2["isect_ids"], 2, tw, th), "adapter offsets two images")


@pytest.mark.parametrize("n,bits", [(1, 40), (4097, 45), (300_001, 64)])
def test_adapter_sort_primitive(dev, n, bits):
    rng = np.random.default_rng(n)
    keys = rng.integers(0, 1 << min(bits, 19), size=n, dtype=np.int64) << max(0, bits - 19)
    ids = rng.integers(0, 1 << 30, size=n, dtype=np.int32)
    sk, si = dev.b200_sort(keys, ids, bits)
    order = np.argsort(keys, kind="stable")
    assert_exact(sk, keys[order], "adapter sort keys")
    assert_exact(si, ids[order], "adapter sort ids")


def test_adapter_rasterize(gs, dev, golden):
    d = golden("chain_cfg1")
    W, H, ts = int(d["width"]), int(d["height"]), int(d["tile_size"])
    bg = np.array([[0.1, 0.2, 0.3]], np.float32)
    inp = dict(means2d=d["proj_means2d"].reshape(1, -1, 2),
               conics=d["proj_conics"].reshape(1, -1, 3), colors=d["colors"],
               opacities=d["opacities"][None], tile_offsets=d["tile_offsets"],
               flatten_ids=d["isect_flatten_ids"], backgrounds=bg)
    a = dev.raster_fwd(width=W, height=H, tile_size=ts, **inp)
    g = gs.rasterize_to_pixels_3dgs_forward({k: T(v) for k, v in inp.items()}, W, H, ts)
    for k in ("render_colors", "render_alphas", "last_ids"):
        assert_exact(a[k], to_np(g[k]), "adapter " + k)
    assert_exact(a["last_ids"], d["rf_last_ids"], "adapter last_ids vs reference")
    rng = np.random.default_rng(9)
    vrc = rng.normal(size=a["render_colors"].shape).astype(np.float32)
    vra = rng.normal(0, 0.1, size=a["render_alphas"].shape).astype(np.float32)
    ab = dev.raster_bwd(width=W, height=H, tile_size=ts, render_alphas=a["render_alphas"],
                        last_ids=a["last_ids"], v_render_colors=vrc, v_render_alphas=vra,
                        absgrad=True, **inp)
    gb = gs.rasterize_to_pixels_3dgs_backward(
        {k: T(v) for k, v in inp.items()},
        {"render_alphas": T(a["render_alphas"]), "last_ids": T(a["last_ids"])},
        {"v_render_colors": T(vrc), "v_render_alphas": T(vra)}, W, H, ts, absgrad=True)
    for k, v in ab.items():
        assert_grad_close(v, to_np(gb[k]), "adapter " + k, atol_frac=1e-5)
