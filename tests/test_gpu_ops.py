"""GPU parity of every operator against the CPU oracle and the golden
fixtures (the reference's own outputs).  Integer results (radii, tile
counts, keys, sort order, offsets, last ids) must be bit-exact on every
entry; float forward values within 1e-5 abs / 1e-4 rel; gradients within
1e-3 rel.

Rasterization decides per pixel x Gaussian whether alpha clears 1/255,
whether it is clamped at 0.99 and whether T(1-alpha) drops to 1e-4.  The
kernels make those decisions exactly as the reference does (its sigma, the
correctly rounded exponential wherever the fast one is within its error of
a threshold), so every pixel is compared, with no exclusions.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from _util import assert_exact, assert_fwd_close, assert_grad_close, to_np

pytestmark = pytest.mark.gpu


def T(x, dev="cuda"):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


# ---------------------------------------------------------------- quat/scale

@pytest.mark.parametrize("triu", [True, False])
@pytest.mark.parametrize("covar,preci", [(True, True), (True, False), (False, True)])
def test_quat_scale_fwd_bwd(gs, oracle, cuda, triu, covar, preci):
    rng = np.random.default_rng(3)
    n = 10_007
    q = rng.normal(size=(n, 4)).astype(np.float32)
    s = np.exp(rng.uniform(-3, 1, size=(n, 3))).astype(np.float32)
    f = gs.quat_scale_to_covar_preci_forward({"quats": T(q), "scales": T(s)}, covar, preci, triu)
    e = oracle.qs2c_fwd(q, s, covar, preci, triu)
    for k in ("covars", "precis"):
        assert tuple(f[k].shape) == e[k].shape
        if e[k].size:
            assert_fwd_close(f[k], e[k], k, atol=1e-5 * max(1.0, np.abs(e[k]).max()))
    shape = (n, 6) if triu else (n, 3, 3)
    vc = rng.normal(size=shape).astype(np.float32) if covar else None
    vp = rng.normal(size=shape).astype(np.float32) if preci else None
    cot = {}
    if covar:
        cot["v_covars"] = T(vc)
    if preci:
        cot["v_precis"] = T(vp)
    b = gs.quat_scale_to_covar_preci_backward({"quats": T(q), "scales": T(s)}, cot, triu)
    eb = oracle.qs2c_bwd(q, s, vc, vp, triu)
    assert_grad_close(b["v_quats"], eb["v_quats"], "v_quats")
    assert_grad_close(b["v_scales"], eb["v_scales"], "v_scales")


def test_quat_scale_golden_and_zero_cotangents(gs, golden, cuda):
    d = golden("ops")
    q, s = T(d["qs_quats"]), T(d["qs_scales"])
    for triu in (0, 1):
        f = gs.quat_scale_to_covar_preci_forward({"quats": q, "scales": s}, True, True, bool(triu))
        assert_fwd_close(f["covars"], d[f"qs_triu{triu}_covars"], "covars golden", atol=1e-4)
        assert_fwd_close(f["precis"], d[f"qs_triu{triu}_precis"], "precis golden", atol=1e-4)
        b = gs.quat_scale_to_covar_preci_backward(
            {"quats": q, "scales": s},
            {"v_covars": T(d[f"qs_triu{triu}_vc"]), "v_precis": T(d[f"qs_triu{triu}_vp"])},
            bool(triu))
        assert_grad_close(b["v_quats"], d[f"qs_triu{triu}_v_quats"], "v_quats golden")
        assert_grad_close(b["v_scales"], d[f"qs_triu{triu}_v_scales"], "v_scales golden")
    z = gs.quat_scale_to_covar_preci_backward({"quats": q, "scales": s}, {}, True)
    assert float(z["v_quats"].abs().max()) == 0.0 and float(z["v_scales"].abs().max()) == 0.0
    e = gs.quat_scale_to_covar_preci_forward({"quats": q[:0], "scales": s[:0]})
    assert tuple(e["covars"].shape) == (0, 6)


# ---------------------------------------------------------------- projection

def _scene_subset(cfg, n, seed=0):
    from gsplat_core import synthetic as S
    sc = getattr(S, cfg)(seed=seed) if cfg != "config3" else S.config3(seed=seed, n=max(n, 10))
    rng = np.random.default_rng(seed + 1)
    idx = np.sort(rng.choice(sc.n, size=min(n, sc.n), replace=False))
    return sc, idx


@pytest.mark.parametrize("cfg,n,use_opac,comp", [
    ("config1", 10_000, False, False), ("config1", 10_000, True, True),
    ("config3", 200_000, False, False), ("config3", 200_000, True, False),
    ("config3", 1_000_000, True, True),
])
def test_projection_fwd_exact(gs, oracle, cuda, cfg, n, use_opac, comp):
    sc, idx = _scene_subset(cfg, n)
    means, quats, scales = sc.means[idx][None], sc.quats[idx][None], sc.scales[idx][None]
    opac = sc.opacities[idx][None] if use_opac else None
    W, H = sc.width, sc.height
    inputs = {"means": T(means), "quats": T(quats), "scales": T(scales),
              "viewmats": T(sc.viewmats[None]), "Ks": T(sc.Ks[None])}
    if use_opac:
        inputs["opacities"] = T(opac)
    g = gs.projection_ewa_3dgs_fused_forward(inputs, W, H, calc_compensations=comp)
    e = oracle.proj_fwd(means, sc.viewmats[None], sc.Ks[None], W, H, quats=quats, scales=scales,
                        opacities=opac, calc_compensations=comp)
    # Compiled without FMA contraction in the reference's operation order,
    # with the correctly rounded log for the opacity-aware extent: every
    # output is bit-identical.
    assert_exact(g["radii"], e["radii"], "radii")
    assert_exact(g["means2d"], e["means2d"], "means2d")
    assert_exact(g["depths"], e["depths"], "depths")
    assert_exact(g["conics"], e["conics"], "conics")
    if comp:
        assert_exact(g["compensations"], e["compensations"], "compensations")
    assert_fwd_close(g["means2d"], e["means2d"], "means2d")
    assert_fwd_close(g["depths"], e["depths"], "depths")
    assert_fwd_close(g["conics"], e["conics"], "conics", atol=1e-5 * max(1, np.abs(e["conics"]).max()))
    if comp:
        assert_fwd_close(g["compensations"], e["compensations"], "compensations")
    else:
        assert tuple(g["compensations"].shape) == (0,)


def test_projection_misaligned_quats(gs, oracle, cuda):
    """Quaternions on a 4-byte (not 16-byte) boundary take the scalar load
    path and give the same bits."""
    sc, idx = _scene_subset("config3", 20_000)
    quats = sc.quats[idx][None]
    buf = torch.zeros(quats.size + 1, dtype=torch.float32, device="cuda")
    buf[1:] = T(quats.ravel())
    q_odd = buf[1:].view(quats.shape)
    assert q_odd.data_ptr() % 16 != 0
    base = {"means": T(sc.means[idx][None]), "scales": T(sc.scales[idx][None]),
            "viewmats": T(sc.viewmats[None]), "Ks": T(sc.Ks[None])}
    a = gs.projection_ewa_3dgs_fused_forward(dict(base, quats=T(quats)), sc.width, sc.height)
    b = gs.projection_ewa_3dgs_fused_forward(dict(base, quats=q_odd), sc.width, sc.height)
    for k in ("radii", "means2d", "depths", "conics"):
        assert torch.equal(a[k], b[k]), k


def test_projection_golden_and_covars(gs, golden, cuda):
    d = golden("ops")
    W, H = int(d["pc_width"]), int(d["pc_height"])
    inputs = {"means": T(d["pc_means"]), "covars": T(d["pc_covars"]),
              "viewmats": T(d["pc_viewmats"]), "Ks": T(d["pc_Ks"])}
    g = gs.projection_ewa_3dgs_fused_forward(inputs, W, H, near_plane=2.4, far_plane=3.9)
    for k in ("radii", "means2d", "depths", "conics"):
        assert_exact(g[k], d["pc_" + k], "golden proj " + k)
    for vm in (True, False):  # without v_viewmats the warp-queue kernel runs
        b = gs.projection_ewa_3dgs_fused_backward(
            inputs, {"radii": g["radii"], "conics": g["conics"]},
            {"v_means2d": T(d["pc_vm2"]), "v_depths": T(d["pc_vd"]), "v_conics": T(d["pc_vco"])},
            W, H, viewmats_requires_grad=vm)
        for k in ("v_means", "v_covars") + (("v_viewmats",) if vm else ()):
            assert_grad_close(b[k], d["pcb_" + k], "golden proj bwd " + k)


@pytest.mark.parametrize("cfg,n,comp,vm", [("config1", 10_000, True, True),
                                           ("config3", 100_000, False, True),
                                           ("config3", 100_000, True, False),
                                           ("config1", 10_000, False, False)])
def test_projection_bwd(gs, oracle, cuda, cfg, n, comp, vm):
    sc, idx = _scene_subset(cfg, n)
    means, quats, scales = sc.means[idx][None], sc.quats[idx][None], sc.scales[idx][None]
    W, H = sc.width, sc.height
    e = oracle.proj_fwd(means, sc.viewmats[None], sc.Ks[None], W, H, quats=quats, scales=scales,
                        calc_compensations=comp)
    rng = np.random.default_rng(9)
    vm2 = rng.normal(size=e["means2d"].shape).astype(np.float32)
    vd = rng.normal(size=e["depths"].shape).astype(np.float32)
    vco = rng.normal(size=e["conics"].shape).astype(np.float32) * 1e-3
    vcp = rng.normal(size=e["depths"].shape).astype(np.float32) if comp else None
    fo = {"radii": T(e["radii"]), "conics": T(e["conics"])}
    cot = {"v_means2d": T(vm2), "v_depths": T(vd), "v_conics": T(vco)}
    if comp:
        fo["compensations"] = T(e["compensations"])
        cot["v_compensations"] = T(vcp)
    b = gs.projection_ewa_3dgs_fused_backward(
        {"means": T(means), "quats": T(quats), "scales": T(scales),
         "viewmats": T(sc.viewmats[None]), "Ks": T(sc.Ks[None])}, fo, cot, W, H,
        viewmats_requires_grad=vm)
    eb = oracle.proj_bwd(means, sc.viewmats[None], sc.Ks[None], W, H, e["radii"], e["conics"],
                         vm2, vd, vco, quats=quats, scales=scales,
                         compensations=e["compensations"] if comp else None,
                         v_compensations=vcp, viewmats_requires_grad=vm)
    for k, v in eb.items():
        assert_grad_close(b[k], v, "proj bwd " + k, atol_frac=1e-4 if k == "v_viewmats" else 1e-5)
    if not vm:
        assert "v_viewmats" not in b


@pytest.mark.parametrize("model", [1, 2])
def test_projection_other_camera_models(gs, oracle, cuda, model):
    """Orthographic / fisheye forward follow metal/gsplat_projection.metal:
    156-201 (the reference CPU path has no counterpart: unpinned)."""
    sc, idx = _scene_subset("config1", 5000)
    means, quats, scales = sc.means[idx][None], sc.quats[idx][None], sc.scales[idx][None]
    K = sc.Ks.copy()
    if model == 1:
        K[:, 0, 0] = K[:, 1, 1] = 60.0
    g = gs.projection_ewa_3dgs_fused_forward(
        {"means": T(means), "quats": T(quats), "scales": T(scales),
         "viewmats": T(sc.viewmats[None]), "Ks": T(K[None])}, sc.width, sc.height,
        camera_model=model)
    e = oracle.proj_fwd(means, sc.viewmats[None], K[None], sc.width, sc.height, quats=quats,
                        scales=scales, camera_model=model)
    diff = (to_np(g["radii"]) != e["radii"]).any(-1)
    assert diff.mean() < 1e-3
    ok = ~diff
    assert (e["radii"][..., 0] > 0).sum() > 100
    assert_fwd_close(to_np(g["means2d"])[ok], e["means2d"][ok], "means2d", atol=1e-3)
    assert_fwd_close(to_np(g["conics"])[ok], e["conics"][ok], "conics",
                     atol=1e-4 * max(1, np.abs(e["conics"]).max()), rtol=1e-3)


def test_projection_errors(gs, cuda):
    m = torch.zeros((1, 4, 3), device=cuda)
    v = torch.eye(4, device=cuda)[None, None]
    K = torch.eye(3, device=cuda)[None, None]
    with pytest.raises(RuntimeError, match="covars or quats"):
        gs.projection_ewa_3dgs_fused_forward({"means": m, "viewmats": v, "Ks": K}, 8, 8)
    with pytest.raises(RuntimeError, match="pinhole only"):
        gs.projection_ewa_3dgs_fused_backward(
            {"means": m, "viewmats": v, "Ks": K, "covars": torch.zeros((1, 4, 6), device=cuda)},
            {"radii": torch.zeros((1, 1, 4, 2), dtype=torch.int32, device=cuda),
             "conics": torch.zeros((1, 1, 4, 3), device=cuda)},
            {"v_means2d": torch.zeros((1, 1, 4, 2), device=cuda),
             "v_depths": torch.zeros((1, 1, 4), device=cuda),
             "v_conics": torch.zeros((1, 1, 4, 3), device=cuda)}, 8, 8, camera_model=1)


# ---------------------------------------------------------------- SH

@pytest.mark.parametrize("deg", [0, 1, 2, 3, 4])
def test_sh_golden(gs, golden, cuda, deg):
    d = golden("ops")
    inputs = {"dirs": T(d["sh_dirs"]), "coeffs": T(d["sh_coeffs"]), "masks": T(d["sh_masks"])}
    c = gs.spherical_harmonics_forward(deg, inputs)
    assert_fwd_close(c, d[f"sh_deg{deg}_colors"], f"sh fwd deg{deg}")
    b = gs.spherical_harmonics_backward(deg, inputs, {"v_colors": T(d["sh_vcol"])})
    assert_grad_close(b["v_coeffs"], d[f"sh_deg{deg}_v_coeffs"], f"sh v_coeffs deg{deg}")
    assert_grad_close(b["v_dirs"], d[f"sh_deg{deg}_v_dirs"], f"sh v_dirs deg{deg}")


@pytest.mark.parametrize("deg,K", [(3, 16), (2, 16), (1, 4), (4, 25)])
def test_sh_large(gs, oracle, cuda, deg, K):
    rng = np.random.default_rng(deg)
    n = 200_003
    dirs = rng.normal(size=(n, 3)).astype(np.float32)
    co = rng.normal(0, 0.3, size=(n, K, 3)).astype(np.float32)
    vc = rng.normal(size=(n, 3)).astype(np.float32)
    c = gs.spherical_harmonics_forward(deg, {"dirs": T(dirs), "coeffs": T(co)})
    assert_fwd_close(c, oracle.sh_fwd(deg, dirs, co), "sh fwd")
    b = gs.spherical_harmonics_backward(deg, {"dirs": T(dirs), "coeffs": T(co)}, {"v_colors": T(vc)},
                                        compute_v_dirs=False)
    eb = oracle.sh_bwd(deg, dirs, co, vc, compute_v_dirs=False)
    assert "v_dirs" not in b
    assert_grad_close(b["v_coeffs"], eb["v_coeffs"], "sh v_coeffs")


@pytest.mark.parametrize("K", [16, 25])
def test_sh_glue_bwd_camera_groups(gs, oracle, cuda, K):
    """The glue backward reading colour cotangents in the interleaved order
    of the camera-sharded step (camera_groups = G: row j G + g is camera j
    of group g) gives the oracle's gradients for the same cameras in
    viewmats order; with zero-cotangent skipping and no radii, as that step
    runs it, on both kernel families."""
    from gsplat_core import pipeline, synthetic as S
    sc, idx = _scene_subset("config3", 40_000)
    means = sc.means[idx]
    rng = np.random.default_rng(7)
    coeffs = (sc.coeffs[idx] if K == 16 else
              rng.normal(0, 0.3, size=(means.shape[0], K, 3)).astype(np.float32))
    G, Cg = 4, 2
    views = S.orbit(G * Cg, 4.0)
    vout = rng.normal(size=(G * Cg, means.shape[0], 3)).astype(np.float32)
    vout[rng.uniform(size=vout.shape[:2]) < 0.5] = 0.0
    perm = [g * Cg + j for j in range(Cg) for g in range(G)]   # row j G + g
    e = oracle.sh_glue_bwd(3, means, views, coeffs, vout, None)
    vm = torch.zeros((means.shape[0], 3), dtype=torch.float32, device="cuda")
    vc = pipeline.sh_colors_backward(3, T(means), T(views), T(coeffs), None, T(vout[perm]), vm,
                                     skip_zero_cotangents=True, camera_groups=G)
    assert_grad_close(vc, e["v_coeffs"], "grouped v_coeffs", atol_frac=1e-5)
    assert_grad_close(vm, e["v_means"], "grouped v_means", atol_frac=1e-5)


@pytest.mark.parametrize("deg,K,misalign", [(3, 16, False), (3, 16, True), (2, 16, False),
                                             (1, 4, False), (0, 4, False), (0, 1, False),
                                             (2, 9, False), (4, 25, False)])
def test_sh_glue(gs, oracle, cuda, deg, K, misalign):
    """Fused colour glue (scanner_points_training_utils.py:1005-1034) against
    the composition restated in the oracle, with and without masks, on both
    kernel families (vectorised rows: K % 4 == 0, 16-byte aligned, degree
    <= 3; warp-staged otherwise)."""
    from gsplat_core import pipeline
    sc, idx = _scene_subset("config3", 50_000)
    means = sc.means[idx]
    rng = np.random.default_rng(2 + deg)
    if K == 16:
        coeffs = sc.coeffs[idx]
    else:
        coeffs = rng.normal(0, 0.3, size=(means.shape[0], K, 3)).astype(np.float32)
        coeffs[:, 0] += 0.5
    views = np.concatenate([sc.viewmats, sc.viewmats @ np.diag([1, 1, 1, 1]).astype(np.float32)])
    views[1, :3, 3] += np.array([0.3, -0.2, 0.5], np.float32)
    masks = rng.uniform(size=(2, means.shape[0])) > 0.3

    def dev_coeffs():
        if not misalign:
            return T(coeffs)
        buf = torch.zeros(coeffs.size + 1, dtype=torch.float32, device="cuda")
        buf[1:] = T(coeffs.ravel())
        return buf[1:].view(coeffs.shape)   # 4-byte aligned only

    for m in (None, masks):
        col = pipeline.sh_colors(deg, T(means), T(views), dev_coeffs(), None if m is None else T(m))
        e = oracle.sh_glue_fwd(deg, means, views, coeffs, m)
        assert_fwd_close(col, e, "glue fwd")
        vout = rng.normal(size=e.shape).astype(np.float32)
        vm0 = rng.normal(size=means.shape).astype(np.float32)
        v_means = T(vm0.copy())
        vco = pipeline.sh_colors_backward(deg, T(means), T(views), dev_coeffs(),
                                          None if m is None else T(m), T(vout), v_means)
        eb = oracle.sh_glue_bwd(deg, means, views, coeffs, vout, m)
        assert_grad_close(vco, eb["v_coeffs"], "glue v_coeffs")
        assert_grad_close(to_np(v_means) - vm0, eb["v_means"], "glue v_means", atol_frac=1e-4)
        # zero cotangents skipped: the same sums
        vz = vout.copy()
        vz[rng.uniform(size=vz.shape[:2]) < 0.4] = 0.0
        v_means = T(vm0.copy())
        vcz = pipeline.sh_colors_backward(deg, T(means), T(views), dev_coeffs(),
                                          None if m is None else T(m), T(vz), v_means,
                                          skip_zero_cotangents=True)
        ez = oracle.sh_glue_bwd(deg, means, views, coeffs, vz, m)
        assert_grad_close(vcz, ez["v_coeffs"], "glue v_coeffs (skip zero)")
        assert_grad_close(to_np(v_means) - vm0, ez["v_means"], "glue v_means (skip zero)",
                          atol_frac=1e-4)


# ---------------------------------------------------------------- intersect

def _isect_inputs(oracle, cfg, n, seed=0):
    sc, idx = _scene_subset(cfg, n, seed)
    e = oracle.proj_fwd(sc.means[idx][None], sc.viewmats[None], sc.Ks[None], sc.width, sc.height,
                        quats=sc.quats[idx][None], scales=sc.scales[idx][None])
    return sc, e["means2d"].reshape(1, -1, 2), e["radii"].reshape(1, -1, 2), e["depths"].reshape(1, -1)


@pytest.mark.parametrize("cfg,n", [("config1", 10_000), ("config3", 300_000)])
@pytest.mark.parametrize("sort", [True, False])
def test_intersect_exact(gs, oracle, cuda, cfg, n, sort):
    sc, m2, rad, dep = _isect_inputs(oracle, cfg, n)
    tw, th = sc.tile_width, sc.tile_height
    g = gs.intersect_tile_forward({"means2d": T(m2), "radii": T(rad), "depths": T(dep)}, 1,
                                  sc.tile_size, tw, th, sort=sort)
    e = oracle.isect_tile(m2, rad, dep, 1, sc.tile_size, tw, th, sort=sort)
    for k in ("tiles_per_gauss", "isect_ids", "flatten_ids"):
        assert_exact(g[k], e[k], k)
    if sort:
        o = gs.intersect_offset_forward(g["isect_ids"], 1, tw, th)
        assert_exact(o, oracle.isect_offset(e["isect_ids"], 1, tw, th), "offsets")


def test_intersect_golden(gs, golden, cuda):
    for name in ("chain_cfg1", "chain_cfg3"):
        d = golden(name)
        W, H, ts = int(d["width"]), int(d["height"]), int(d["tile_size"])
        tw, th = (W + ts - 1) // ts, (H + ts - 1) // ts
        inp = {"means2d": T(d["proj_means2d"].reshape(1, -1, 2)),
               "radii": T(d["proj_radii"].reshape(1, -1, 2)),
               "depths": T(d["proj_depths"].reshape(1, -1))}
        g = gs.intersect_tile_forward(inp, 1, ts, tw, th, sort=True)
        for k in ("tiles_per_gauss", "isect_ids", "flatten_ids"):
            assert_exact(g[k].reshape(-1), d["isect_" + k].reshape(-1), f"{name} {k}")
        u = gs.intersect_tile_forward(inp, 1, ts, tw, th, sort=False)
        assert_exact(u["isect_ids"], d["isect_unsorted_isect_ids"], f"{name} unsorted")
        o = gs.intersect_offset_forward(g["isect_ids"], 1, tw, th)
        assert_exact(o, d["tile_offsets"], f"{name} offsets")


def test_intersect_known_answers(gs, cuda):
    """gsplat_core/test/test.cpp:653-1065 through the GPU path."""
    m2 = T(np.array([[[50, 50], [20, 20], [8, 8]]], np.float32))
    rad = T(np.array([[[5, 5], [10, 10], [0, 0]]], np.int32))
    dep = T(np.array([[0.5, 1.0, 2.0]], np.float32))
    r = gs.intersect_tile_forward({"means2d": m2, "radii": rad, "depths": dep}, 1, 16, 4, 4)
    assert to_np(r["tiles_per_gauss"]).tolist() == [[4, 4, 0]]
    assert to_np(r["isect_ids"]).tolist() == [(t << 32) | 0x3F800000 for t in (0, 1, 4, 5)] + \
        [(t << 32) | 0x3F000000 for t in (10, 11, 14, 15)]
    assert to_np(r["flatten_ids"]).tolist() == [1, 1, 1, 1, 0, 0, 0, 0]
    o = gs.intersect_offset_forward(r["isect_ids"], 1, 4, 4)
    assert to_np(o).ravel().tolist() == [0, 1, 2, 2, 2, 3, 4, 4, 4, 4, 4, 5, 6, 6, 6, 7]


def test_intersect_multi_image_and_empty(gs, oracle, cuda):
    rng = np.random.default_rng(4)
    I, N = 3, 5000
    m2 = rng.uniform(-20, 280, size=(I, N, 2)).astype(np.float32)
    rad = rng.integers(-1, 30, size=(I, N, 2)).astype(np.int32)
    dep = rng.uniform(0.1, 50, size=(I, N)).astype(np.float32)
    dep[0, :100] = dep[0, 100]  # ties: stability decides the order
    g = gs.intersect_tile_forward({"means2d": T(m2), "radii": T(rad), "depths": T(dep)}, I, 8, 32, 32)
    e = oracle.isect_tile(m2, rad, dep, I, 8, 32, 32)
    for k in ("tiles_per_gauss", "isect_ids", "flatten_ids"):
        assert_exact(g[k], e[k], k)
    assert_exact(gs.intersect_offset_forward(g["isect_ids"], I, 32, 32),
                 oracle.isect_offset(e["isect_ids"], I, 32, 32), "offsets")
    z = gs.intersect_tile_forward({"means2d": T(m2), "radii": T(np.zeros_like(rad)),
                                   "depths": T(dep)}, I, 8, 32, 32)
    assert z["isect_ids"].numel() == 0 and z["flatten_ids"].numel() == 0
    oz = gs.intersect_offset_forward(z["isect_ids"], I, 32, 32)
    assert int(oz.abs().max()) == 0


def test_intersect_sorted_depth_bits(gs, oracle, cuda):
    """The depth-first sorted encode orders by the raw depth bits like the
    64-bit key sort: negative depths and -0.0 (sign bit set) after the
    positives, heavy ties across many element-sort tiles, two images."""
    rng = np.random.default_rng(9)
    I, N = 2, 150_001
    m2 = rng.uniform(-40, 700, size=(I, N, 2)).astype(np.float32)
    rad = rng.integers(0, 24, size=(I, N, 2)).astype(np.int32)
    dep = rng.choice(np.array([0.5, 1.0, 2.0, -1.0, 0.0, -0.0, 3.25], np.float32), size=(I, N))
    dep[:, ::7] = rng.uniform(-5, 5, size=dep[:, ::7].shape).astype(np.float32)
    g = gs.intersect_tile_forward({"means2d": T(m2), "radii": T(rad), "depths": T(dep)}, I, 16,
                                  42, 40)
    e = oracle.isect_tile(m2, rad, dep, I, 16, 42, 40)
    for k in ("tiles_per_gauss", "isect_ids", "flatten_ids"):
        assert_exact(g[k], e[k], k)
    # the same as encode followed by the plain key sort
    u = gs.intersect_tile_forward({"means2d": T(m2), "radii": T(rad), "depths": T(dep)}, I, 16,
                                  42, 40, sort=False)
    tb = gs.floor_log2_plus_one(42 * 40)
    ib = gs.floor_log2_plus_one(I)
    sk, sv = gs.intersect_tile_sort(u["isect_ids"], u["flatten_ids"], 32 + tb + ib)
    assert torch.equal(sk, g["isect_ids"]) and torch.equal(sv, g["flatten_ids"])


def test_intersect_binned_offsets_bands_and_fallback(gs, oracle, cuda):
    """The binned encode (the sort=True path) also writes the tile offsets;
    over a window of tile rows it gives exactly that window's part of the
    full sorted list and its offsets; the depth-first sorted encode (the
    path for tile grids past 16-bit coordinates) gives the same lists."""
    import ctypes as ct
    from gsplat_core import _gsplat_core as G, _lib
    from gsplat_core._lib import IsectParams
    lib = _lib.load()
    rng = np.random.default_rng(11)
    I, N, ts, tw, th = 2, 40_000, 16, 37, 23
    m2 = rng.uniform(-30, tw * ts + 30, size=(I, N, 2)).astype(np.float32)
    rad = rng.integers(-2, 40, size=(I, N, 2)).astype(np.int32)
    dep = rng.uniform(0.1, 20, size=(I, N)).astype(np.float32)
    dep[:, ::5] = dep[:, 1:2]  # ties: element order decides
    e = oracle.isect_tile(m2, rad, dep, I, ts, tw, th)
    eo = oracle.isect_offset(e["isect_ids"], I, tw, th)
    tpg, m, bins = G.intersect_tile_count_totals(T(m2), T(rad), I, ts, tw, th)
    assert m == len(e["isect_ids"]) and 0 < bins <= m
    offs = torch.full((I, th, tw), -1, dtype=torch.int32, device="cuda")
    ids, fids = G.intersect_tile_encode_binned(T(m2), T(rad), T(dep), I, ts, tw, th, m, bins, offs)
    assert_exact(ids, e["isect_ids"], "binned isect_ids")
    assert_exact(fids, e["flatten_ids"], "binned flatten_ids")
    assert_exact(offs, eo, "binned tile offsets")
    sid, sfid = G.intersect_tile_encode_sorted(T(m2), T(rad), T(dep), tpg, I, ts, tw, th, m)
    assert torch.equal(sid, ids) and torch.equal(sfid, fids)
    # tile rows [y0, y1) only
    y0, y1 = 5, 14
    tb = gs.floor_log2_plus_one(tw * th)
    tile = (e["isect_ids"] >> 32) & ((1 << tb) - 1)
    keep = (tile // tw >= y0) & (tile // tw < y1)
    bid, bfid = e["isect_ids"][keep], e["flatten_ids"][keep]
    keys = np.array([(i << tb) | (y * tw + x) for i in range(I) for y in range(y0, y1)
                     for x in range(tw)], np.int64)
    bofs = np.searchsorted(bid >> 32, keys, side="left").astype(np.int32)
    p = IsectParams(I, N, ts, tw, th, y0, y1)
    s = ct.c_void_p(torch.cuda.current_stream().cuda_stream)
    P = lambda t: ct.c_void_p(t.data_ptr())  # noqa: E731
    tot = torch.zeros(2, dtype=torch.int64, device="cuda")
    tpg_b = torch.empty((I, N), dtype=torch.int32, device="cuda")
    dm2, drad, ddep = T(m2), T(rad), T(dep)
    assert lib.gs_isect_tile_count_totals(ct.byref(p), P(dm2), P(drad), P(tpg_b), P(tot), s) == 0
    mb, binsb = (int(v) for v in tot.tolist())
    assert mb == len(bid)
    ob = torch.full((I, y1 - y0, tw), -1, dtype=torch.int32, device="cuda")
    oid = torch.empty(mb, dtype=torch.int64, device="cuda")
    ofid = torch.empty(mb, dtype=torch.int32, device="cuda")
    ws = torch.empty(lib.gs_isect_tile_encode_binned_workspace_size(ct.byref(p), binsb),
                     dtype=torch.uint8, device="cuda")
    assert lib.gs_isect_tile_encode_binned(ct.byref(p), P(dm2), P(drad), P(ddep), mb, binsb,
                                           P(oid), P(ofid), P(ob), P(ws), ws.numel(), s) == 0
    assert lib.gs_isect_tile_encode_binned_check(binsb, P(ws), s) == 0
    assert_exact(oid, bid, "band isect_ids")
    assert_exact(ofid, bfid, "band flatten_ids")
    assert_exact(ob.reshape(-1), bofs, "band tile offsets")
    # the caller's promise of positive depths (31-bit depth field in the
    # entry keys) gives the same lists
    q = IsectParams(I, N, ts, tw, th, 0, 0, 0, 1)
    assert lib.gs_isect_tile_count_totals(ct.byref(q), P(dm2), P(drad), P(tpg_b), P(tot), s) == 0
    mq, binsq = (int(v) for v in tot.tolist())
    qid = torch.empty(mq, dtype=torch.int64, device="cuda")
    qfid = torch.empty(mq, dtype=torch.int32, device="cuda")
    ws = torch.empty(lib.gs_isect_tile_encode_binned_workspace_size(ct.byref(q), binsq),
                     dtype=torch.uint8, device="cuda")
    assert lib.gs_isect_tile_encode_binned(ct.byref(q), P(dm2), P(drad), P(ddep), mq, binsq,
                                           P(qid), P(qfid), None, P(ws), ws.numel(), s) == 0
    assert_exact(qid, e["isect_ids"], "positive-depth isect_ids")
    assert_exact(qfid, e["flatten_ids"], "positive-depth flatten_ids")


def test_sort_error_words_clear(gs, cuda):
    """The bounded look-back waits of a sort end normally: the error word the
    check entry points read stays clear (GS_OK) after real sorts."""
    import ctypes as ct
    from gsplat_core import _lib
    lib = _lib.load()
    rng = np.random.default_rng(3)
    n = 3_000_001
    keys = T(rng.integers(0, 1 << 40, size=n).astype(np.int64))
    vals = T(np.arange(n, dtype=np.int32))
    ok, ov = torch.empty_like(keys), torch.empty_like(vals)
    ws = torch.empty(lib.gs_isect_sort_workspace_size(n), dtype=torch.uint8, device="cuda")
    s = ct.c_void_p(torch.cuda.current_stream().cuda_stream)
    P = lambda t: ct.c_void_p(t.data_ptr())  # noqa: E731
    assert lib.gs_isect_sort(n, 40, P(keys), P(vals), P(ok), P(ov), P(ws), ws.numel(), s) == 0
    assert lib.gs_isect_sort_check(n, P(ws), s) == 0
    assert bool((ok[1:] >= ok[:-1]).all())


def test_sort_wait_gives_up_and_reports(gs, cuda):
    """The give-up path of the bounded look-back wait: a radix pass whose
    second tile runs alone waits 16 polls for the first, which never
    publishes, then raises the error word and finishes; the check entry
    reports GS_ERR_DEVICE (and clears after a normal sort in the same
    workspace).  Its outputs stay in range: the second tile's keys land at
    places inside the arrays, the rest keeps the fill."""
    import ctypes as ct
    from gsplat_core import _lib
    lib = _lib.load()
    rng = np.random.default_rng(5)
    n = 6000
    keys = T(rng.integers(0, 1 << 12, size=n).astype(np.int64))
    vals = T(np.arange(n, dtype=np.int32))
    ok = torch.full_like(keys, -7)
    ov = torch.full_like(vals, -7)
    ws = torch.empty(lib.gs_isect_sort_workspace_size(n), dtype=torch.uint8, device="cuda")
    s = ct.c_void_p(torch.cuda.current_stream().cuda_stream)
    P = lambda t: ct.c_void_p(t.data_ptr())  # noqa: E731
    assert lib.gs_isect_sort_wait_selftest(n, P(keys), P(vals), P(ok), P(ov), P(ws), ws.numel(),
                                           16, s) == 0, lib.gs_last_error()
    assert lib.gs_isect_sort_check(n, P(ws), s) == 6  # GS_ERR_DEVICE
    assert b"gave up" in lib.gs_last_error()
    torch.cuda.synchronize()
    # the 1904 keys of tile 1 were written, each an input key of tile 1
    written = (ov != -7).cpu().numpy()
    assert written.sum() == n - 4096
    assert set(to_np(ov)[written].tolist()) == set(range(4096, n))
    # bad arguments are refused before any launch
    assert lib.gs_isect_sort_wait_selftest(4096, P(keys), P(vals), P(ok), P(ov), P(ws),
                                           ws.numel(), 16, s) == 1
    assert lib.gs_isect_sort_wait_selftest(n, P(keys), P(vals), P(ok), P(ov), P(ws),
                                           ws.numel(), 5000, s) == 1
    # a normal sort in the same workspace clears the word
    assert lib.gs_isect_sort(n, 44, P(keys), P(vals), P(ok), P(ov), P(ws), ws.numel(), s) == 0
    assert lib.gs_isect_sort_check(n, P(ws), s) == 0


@pytest.mark.parametrize("n", [1, 31, 4095, 4096, 4097, 100_000, 1_000_003])
@pytest.mark.parametrize("bits", [40, 46, 64])
def test_sort_stable_exact(gs, oracle, cuda, n, bits):
    """The radix sort against a stable merge sort: random keys with many
    duplicates (stability), tile boundaries, and the 64-bit signed order."""
    rng = np.random.default_rng(n + bits)
    hi_bits = bits - 32
    keys = (rng.integers(0, 1 << min(hi_bits, 20), size=n).astype(np.int64) << 32) | \
        rng.integers(0, 64, size=n).astype(np.int64)
    if bits == 64:
        sign = rng.uniform(size=n) < 0.5
        keys = keys | (rng.integers(0, 1 << 30, size=n).astype(np.int64) << 33)
        keys[sign] = -keys[sign]
    vals = np.arange(n, dtype=np.int32)
    gk, gv = gs.intersect_tile_sort(T(keys), T(vals), bits)
    ek, ev = oracle.isect_sort(keys, vals)
    assert_exact(gk, ek, "keys")
    assert_exact(gv, ev, "values (stability)")


# ---------------------------------------------------------------- rasterize

def _raster_case(oracle, name, d, channels=3):
    W, H, ts = int(d["width"]), int(d["height"]), int(d["tile_size"])
    colors = d["colors"]
    if channels != 3:
        rng = np.random.default_rng(channels)
        colors = rng.uniform(0, 1, size=colors.shape[:-1] + (channels,)).astype(np.float32)
    bg = np.linspace(0.1, 0.3, channels, dtype=np.float32)[None]
    inp = dict(means2d=d["proj_means2d"].reshape(1, -1, 2), conics=d["proj_conics"].reshape(1, -1, 3),
               colors=colors, opacities=d["opacities"][None], tile_offsets=d["tile_offsets"],
               flatten_ids=d["isect_flatten_ids"], backgrounds=bg)
    return W, H, ts, inp


@pytest.mark.parametrize("name", ["chain_cfg1", "chain_cfg3"])
@pytest.mark.parametrize("channels", [3, 1, 4, 5])
def test_rasterize_fwd_bwd(gs, oracle, golden, cuda, name, channels):
    d = golden(name)
    W, H, ts, inp = _raster_case(oracle, name, d, channels)
    e = oracle.raster_fwd(width=W, height=H, tile_size=ts, **inp)
    g = gs.rasterize_to_pixels_3dgs_forward({k: T(v) for k, v in inp.items()}, W, H, ts)
    assert_exact(to_np(g["last_ids"]), e["last_ids"], "last_ids")
    assert_fwd_close(to_np(g["render_alphas"]), e["render_alphas"], "alphas")
    assert_fwd_close(to_np(g["render_colors"]), e["render_colors"], "colors")
    if channels == 3:
        assert_exact(to_np(g["last_ids"]), d["rf_last_ids"], "last_ids vs golden")
        assert_fwd_close(to_np(g["render_colors"]), d["rf_render_colors"], "colors vs golden")
    # Backward from the oracle's forward state, every pixel driven.
    vrc = np.random.default_rng(5).normal(size=e["render_colors"].shape).astype(np.float32)
    vra = np.random.default_rng(6).normal(0, 0.1, size=e["render_alphas"].shape).astype(np.float32)
    fo = {"render_alphas": e["render_alphas"], "last_ids": e["last_ids"]}
    b = gs.rasterize_to_pixels_3dgs_backward(
        {k: T(v) for k, v in inp.items()}, {k: T(v) for k, v in fo.items()},
        {"v_render_colors": T(vrc), "v_render_alphas": T(vra)}, W, H, ts, absgrad=True)
    eb = oracle.raster_bwd(width=W, height=H, tile_size=ts, render_alphas=e["render_alphas"],
                           last_ids=e["last_ids"], v_render_colors=vrc, v_render_alphas=vra,
                           absgrad=True, **inp)
    for k, v in eb.items():
        assert_grad_close(b[k], v, f"{name} {k}", atol_frac=1e-4)


def test_rasterize_known_answers_and_masks(gs, cuda):
    """gsplat_core/test/test.cpp:1067-1271 through the GPU path."""
    base = {"means2d": T(np.array([[[1.0, 1.0]]], np.float32)),
            "conics": T(np.array([[[1.0, 0.0, 1.0]]], np.float32)),
            "colors": T(np.array([[[1.0, 0.0, 0.0]]], np.float32)),
            "opacities": T(np.array([[0.5]], np.float32)),
            "backgrounds": T(np.array([[0.1, 0.2, 0.3]], np.float32)),
            "flatten_ids": T(np.array([0], np.int32))}
    a = 0.5 * np.exp(-0.25)
    Tt = 1 - a
    r = gs.rasterize_to_pixels_3dgs_forward(dict(base, tile_offsets=T(np.zeros((1, 1, 1), np.int32))), 2, 2, 2)
    assert np.allclose(to_np(r["render_alphas"]).ravel(), a, atol=1e-5)
    assert np.allclose(to_np(r["render_colors"]).reshape(4, 3), [a + Tt * .1, Tt * .2, Tt * .3], atol=1e-5)
    assert to_np(r["last_ids"]).ravel().tolist() == [0] * 4
    rm = gs.rasterize_to_pixels_3dgs_forward(
        dict(base, tile_offsets=T(np.array([[[0, 1]]], np.int32)), masks=T(np.array([[[True, False]]]))),
        4, 2, 2)
    al = to_np(rm["render_alphas"]).reshape(2, 4)
    assert np.allclose(al[:, :2], a, atol=1e-5) and np.allclose(al[:, 2:], 0)
    assert np.allclose(to_np(rm["render_colors"]).reshape(2, 4, 3)[:, 2:], [.1, .2, .3], atol=1e-6)


def test_rasterize_masks_backward(gs, oracle, golden, cuda):
    d = golden("chain_cfg1")
    W, H, ts, inp = _raster_case(oracle, "chain_cfg1", d)
    masks = np.random.default_rng(8).uniform(size=d["tile_offsets"].shape) > 0.3
    inp = dict(inp, masks=masks)
    e = oracle.raster_fwd(width=W, height=H, tile_size=ts, **inp)
    g = gs.rasterize_to_pixels_3dgs_forward({k: T(v) for k, v in inp.items()}, W, H, ts)
    assert_exact(to_np(g["last_ids"]), e["last_ids"], "masked last_ids")
    assert_fwd_close(to_np(g["render_colors"]), e["render_colors"], "masked colors")
    vrc = np.random.default_rng(5).normal(size=e["render_colors"].shape).astype(np.float32)
    vra = np.zeros(e["render_alphas"].shape, np.float32)
    b = gs.rasterize_to_pixels_3dgs_backward(
        {k: T(v) for k, v in inp.items()},
        {"render_alphas": T(e["render_alphas"]), "last_ids": T(e["last_ids"])},
        {"v_render_colors": T(vrc), "v_render_alphas": T(vra)}, W, H, ts)
    eb = oracle.raster_bwd(width=W, height=H, tile_size=ts, render_alphas=e["render_alphas"],
                           last_ids=e["last_ids"], v_render_colors=vrc, v_render_alphas=vra, **inp)
    for k, v in eb.items():
        assert_grad_close(b[k], v, "masked " + k, atol_frac=1e-4)


def test_rasterize_tile_cull_boundary(gs, oracle, cuda):
    """The 16x16 rasterizer drops a Gaussian from a tile only when no pixel
    centre of the tile can reach alpha >= 1/255.  Gaussians tuned to peak
    just above / below the threshold inside the tile (thin, rotated, far
    outside and inside it), one per 16x16 image, must render exactly as the
    oracle renders them."""
    rng = np.random.default_rng(21)
    thr = 1.0 / 255.0
    px = np.arange(16) + 0.5
    means, conics, opac, above = [], [], [], []
    while len(means) < 3000:
        th = rng.uniform(0, np.pi)
        s1 = np.exp(rng.uniform(np.log(0.3), np.log(25.0)))
        s2 = s1 / np.exp(rng.uniform(0, np.log(60.0)))
        R = np.array([[np.cos(th), -np.sin(th)], [np.sin(th), np.cos(th)]])
        cov = R @ np.diag([s1 * s1, s2 * s2]) @ R.T
        inv = np.linalg.inv(cov)
        a, b, c = inv[0, 0], inv[0, 1], inv[1, 1]
        m = rng.uniform(-40, 56, size=2)
        dx = m[0] - px[None, :]
        dy = m[1] - px[:, None]
        smin = (0.5 * (a * dx * dx + c * dy * dy) + b * dx * dy).min()
        d = rng.uniform(2e-3, 0.1) * (1 if rng.uniform() < 0.5 else -1)
        if smin > 5.4:
            continue
        o = thr * (1 + d) * np.exp(smin)
        if o > 0.9:
            continue
        means.append(m)
        conics.append([a, b, c])
        opac.append(o)
        above.append(d > 0)
    I = len(means)
    inp = dict(means2d=np.array(means, np.float32).reshape(I, 1, 2),
               conics=np.array(conics, np.float32).reshape(I, 1, 3),
               colors=rng.uniform(0, 1, size=(I, 1, 3)).astype(np.float32),
               opacities=np.array(opac, np.float32).reshape(I, 1),
               tile_offsets=np.arange(I, dtype=np.int32).reshape(I, 1, 1),
               flatten_ids=np.arange(I, dtype=np.int32))
    e = oracle.raster_fwd(width=16, height=16, tile_size=16, **inp)
    g = gs.rasterize_to_pixels_3dgs_forward({k: T(v) for k, v in inp.items()}, 16, 16, 16)
    assert_exact(to_np(g["last_ids"]), e["last_ids"], "last_ids")
    ga = to_np(g["render_alphas"])[..., 0]
    assert_fwd_close(ga, e["render_alphas"][..., 0], "alphas")
    hit = ga.reshape(I, -1).max(1) > 0
    assert np.array_equal(hit, np.array(above)), "a Gaussian reaching the threshold was dropped"
    vrc = rng.normal(size=e["render_colors"].shape).astype(np.float32)
    vra = rng.normal(0, 0.1, size=e["render_alphas"].shape).astype(np.float32)
    b = gs.rasterize_to_pixels_3dgs_backward(
        {k: T(v) for k, v in inp.items()},
        {"render_alphas": T(e["render_alphas"]), "last_ids": T(e["last_ids"])},
        {"v_render_colors": T(vrc), "v_render_alphas": T(vra)}, 16, 16, 16)
    eb = oracle.raster_bwd(width=16, height=16, tile_size=16, render_alphas=e["render_alphas"],
                           last_ids=e["last_ids"], v_render_colors=vrc, v_render_alphas=vra, **inp)
    for k, v in eb.items():
        assert_grad_close(b[k], v, f"cull {k}", atol_frac=1e-4)


def _threshold_cases(seed=31, per_kind=700):
    """One 16x16 image per case, one tile, a short list of Gaussians whose
    decisions at pixel (7, 9) sit within a few ulps of a threshold, computed
    with the C library's expf and float32 arithmetic in the reference's
    order: alpha against 1/255, o e^-sigma against the 0.99 clamp, and
    T (1 - alpha) against 1e-4 (with exact and with inexact exponentials)."""
    import ctypes
    libm = ctypes.CDLL("libm.so.6")
    libm.expf.restype = ctypes.c_float
    libm.expf.argtypes = [ctypes.c_float]
    f = np.float32
    expf = lambda x: f(libm.expf(f(x)))  # noqa: E731
    rng = np.random.default_rng(seed)
    px, py = f(7.5), f(9.5)

    def sigma(m, c):
        dx, dy = f(m[0]) - px, f(m[1]) - py
        return f(0.5) * (c[0] * dx * dx + c[2] * dy * dy) + c[1] * dx * dy

    def conic(scale):
        th = rng.uniform(0, np.pi)
        s1 = scale
        s2 = s1 / rng.uniform(1, 8)
        R = np.array([[np.cos(th), -np.sin(th)], [np.sin(th), np.cos(th)]])
        inv = np.linalg.inv(R @ np.diag([s1 * s1, s2 * s2]) @ R.T)
        return np.array([inv[0, 0], inv[0, 1], inv[1, 1]], np.float32)

    def nudge(v, k):   # k ulps away
        return (np.array([v], np.float32).view(np.int32) + np.int32(k)).view(np.float32)[0]

    cases = []
    for i in range(per_kind):            # alpha against 1/255
        c = conic(rng.uniform(1.0, 6.0))
        m = np.array([7.5, 9.5], np.float32) + rng.uniform(-6, 6, 2).astype(np.float32)
        s = sigma(m, c)
        e = expf(-s)
        if not (0 <= s < 5.0):
            continue
        o = f(f(1.0 / 255.0) / e)
        o = nudge(o, int(rng.integers(-3, 4)))
        if o >= 1:
            continue
        cases.append(([m], [c], [o]))
    for i in range(per_kind):            # o e^-sigma against the 0.99 clamp
        c = conic(rng.uniform(2.0, 6.0))
        m = np.array([7.5, 9.5], np.float32) + rng.uniform(-0.2, 0.2, 2).astype(np.float32)
        s = sigma(m, c)
        e = expf(-s)
        o = nudge(f(f(0.99) / e), int(rng.integers(-3, 4)))
        if not (0 <= s and o <= 1):
            continue
        cases.append(([m], [c], [o]))
    for exact_exp in (True, False):      # T (1 - alpha) against 1e-4
        for i in range(per_kind):
            k = int(rng.integers(4, 12))
            ms, cs, os_ = [], [], []
            T = f(1.0)
            for j in range(k - 1):
                c = conic(rng.uniform(3.0, 8.0))
                m = (np.array([7.5, 9.5], np.float32) if exact_exp else
                     np.array([7.5, 9.5], np.float32) + rng.uniform(-1, 1, 2).astype(np.float32))
                o = f(rng.uniform(0.3, 0.8))
                a = min(f(0.99), o * expf(-sigma(m, c)))
                if sigma(m, c) < 0 or a < f(1 / 255):
                    continue
                nT = T * (f(1) - a)
                if nT <= f(2e-4):
                    break
                T = nT
                ms.append(m); cs.append(c); os_.append(o)
            c = conic(rng.uniform(3.0, 8.0))
            m = (np.array([7.5, 9.5], np.float32) if exact_exp else
                 np.array([7.5, 9.5], np.float32) + rng.uniform(-1, 1, 2).astype(np.float32))
            e = expf(-sigma(m, c))
            need = (1.0 - 1e-4 / float(T)) / float(e)
            if not (0.02 < need < 0.97):
                continue
            o = nudge(f(need), int(rng.integers(-4, 5)))
            ms.append(m); cs.append(c); os_.append(o)
            cases.append((ms, cs, os_))
    return cases


def _threshold_inputs(channels):
    cases = _threshold_cases()
    I = len(cases)
    N = max(len(c[2]) for c in cases)
    rng = np.random.default_rng(32)
    means = np.zeros((I, N, 2), np.float32)
    conics = np.tile(np.array([1, 0, 1], np.float32), (I, N, 1))
    opac = np.zeros((I, N), np.float32)
    fids, offs = [], []
    for i, (ms, cs, os_) in enumerate(cases):
        offs.append(len(fids))
        for j in range(len(os_)):
            means[i, j], conics[i, j], opac[i, j] = ms[j], cs[j], os_[j]
            fids.append(i * N + j)
    inp = dict(means2d=means, conics=conics, opacities=opac,
               colors=rng.uniform(0, 1, size=(I, N, channels)).astype(np.float32),
               tile_offsets=np.array(offs, np.int32).reshape(I, 1, 1),
               flatten_ids=np.array(fids, np.int32),
               backgrounds=np.tile(np.linspace(0.1, 0.3, channels, dtype=np.float32), (I, 1)))
    return cases, offs, inp


@pytest.mark.parametrize("channels", [3, 5])
def test_rasterize_threshold_decisions_exact(gs, oracle, cuda, channels):
    """Decisions within a few ulps of 1/255, 0.99 and 1e-4 (16x16 kernels
    with 3 channels, the generic kernels with 5): last ids bit for bit,
    renders and gradients as the oracle's on every pixel; the cases fall on
    both sides of each threshold."""
    cases, offs, inp = _threshold_inputs(channels)
    rng = np.random.default_rng(33)
    e = oracle.raster_fwd(width=16, height=16, tile_size=16, **inp)
    # both outcomes occur at the target pixel
    lid = e["last_ids"][:, 9, 7] - np.array(offs)
    nk = np.array([len(c[2]) for c in cases])
    alpha_p = e["render_alphas"][:, 9, 7, 0]
    assert (alpha_p == 0).any() and (alpha_p > 0).any()
    assert (lid == nk - 1).any() and (lid == nk - 2).any()
    g = gs.rasterize_to_pixels_3dgs_forward({k: T(v) for k, v in inp.items()}, 16, 16, 16)
    assert_exact(to_np(g["last_ids"]), e["last_ids"], "last_ids")
    assert_fwd_close(to_np(g["render_alphas"]), e["render_alphas"], "alphas")
    assert_fwd_close(to_np(g["render_colors"]), e["render_colors"], "colors")
    vrc = rng.normal(size=e["render_colors"].shape).astype(np.float32)
    vra = rng.normal(0, 0.1, size=e["render_alphas"].shape).astype(np.float32)
    b = gs.rasterize_to_pixels_3dgs_backward(
        {k: T(v) for k, v in inp.items()},
        {"render_alphas": T(e["render_alphas"]), "last_ids": T(e["last_ids"])},
        {"v_render_colors": T(vrc), "v_render_alphas": T(vra)}, 16, 16, 16, absgrad=True)
    eb = oracle.raster_bwd(width=16, height=16, tile_size=16, render_alphas=e["render_alphas"],
                           last_ids=e["last_ids"], v_render_colors=vrc, v_render_alphas=vra,
                           absgrad=True, **inp)
    for k, v in eb.items():
        assert_grad_close(b[k], v, f"threshold {k}", atol_frac=1e-4)


def _length_bucket(x):
    """The tile scheduler's cost bucket: 8 floor(log2 x) + the next three
    bits of x, + 1 (0 for x <= 0)."""
    x = np.asarray(x, np.int64)
    out = np.zeros(x.shape, np.int64)
    nz = x > 0
    lz = np.floor(np.log2(x[nz])).astype(np.int64)
    frac = np.where(lz >= 3, (x[nz] >> np.maximum(lz - 3, 0)) & 7,
                    (x[nz] << np.maximum(3 - lz, 0)) & 7)
    out[nz] = np.minimum(255, lz * 8 + frac + 1)
    return out


@pytest.mark.parametrize("I,tw,th", [(1, 82, 53), (3, 37, 23), (1, 1, 1)])
def test_raster_tile_order(gs, cuda, I, tw, th):
    """The rasterizers' tile schedule is a permutation of the slots in
    non-increasing cost bucket: by list length from the offsets, or by the
    given per-tile costs."""
    import ctypes as ct
    from gsplat_core import _lib
    lib = _lib.load()
    rng = np.random.default_rng(I * 1000 + tw)
    n = I * tw * th
    lens = rng.integers(0, 6000, size=n).astype(np.int64)
    lens[::5] = 0
    lens[1::7] = rng.integers(0, 8, size=lens[1::7].shape)
    offs = np.concatenate([[0], np.cumsum(lens)[:-1]]).astype(np.int32)
    m = int(lens.sum())
    rp = _lib.RasterParams(I, 10, 3, tw * 16, th * 16, 16, tw, th, m, 0, 0, 0)
    s = ct.c_void_p(torch.cuda.current_stream().cuda_stream)
    P = lambda t: ct.c_void_p(t.data_ptr())  # noqa: E731
    order = torch.full((n,), -1, dtype=torch.int32, device="cuda")
    assert lib.gs_raster_tile_order(ct.byref(rp), P(T(offs)), None, P(order), s) == 0
    o = to_np(order).astype(np.int64)
    assert np.array_equal(np.sort(o), np.arange(n))
    b = _length_bucket(lens[o])
    assert np.all(b[1:] <= b[:-1])
    cost = rng.integers(0, 500, size=n).astype(np.int32)
    assert lib.gs_raster_tile_order(ct.byref(rp), None, P(T(cost)), P(order), s) == 0
    o = to_np(order).astype(np.int64)
    assert np.array_equal(np.sort(o), np.arange(n))
    b = _length_bucket(cost[o])
    assert np.all(b[1:] <= b[:-1])


def test_rasterize_fwd_tile_cost_and_ordered_backward(gs, oracle, golden, cuda):
    """The forward's per-tile cost record (the list entries its pixels walk)
    matches the oracle's last ids, and forward / backward run in the
    schedules it gives produce the same images and gradients."""
    import ctypes as ct
    from gsplat_core import _lib
    lib = _lib.load()
    d = golden("chain_cfg3")
    W, H, ts, inp = _raster_case(oracle, "chain_cfg3", d)
    e = oracle.raster_fwd(width=W, height=H, tile_size=ts, **inp)
    dev = {k: T(v) for k, v in inp.items()}
    th, tw = inp["tile_offsets"].shape[-2:]
    n = tw * th
    m = int(inp["flatten_ids"].size)
    N = inp["means2d"].shape[1]
    s = ct.c_void_p(torch.cuda.current_stream().cuda_stream)
    P = lambda t: ct.c_void_p(t.data_ptr()) if t is not None else None  # noqa: E731
    order = torch.empty((n,), dtype=torch.int32, device="cuda")
    cost = torch.full((n,), -7, dtype=torch.int32, device="cuda")
    rp = _lib.RasterParams(1, N, 3, W, H, ts, tw, th, m, 1, 0, 0)
    rp.tile_order = P(order)
    rp.tile_cost = P(cost)
    assert lib.gs_raster_tile_order(ct.byref(rp), P(dev["tile_offsets"]), None, P(order), s) == 0
    rc = torch.empty((1, H, W, 3), device="cuda")
    ra = torch.empty((1, H, W, 1), device="cuda")
    li = torch.empty((1, H, W), dtype=torch.int32, device="cuda")
    assert lib.gs_rasterize_fwd(ct.byref(rp), P(dev["means2d"]), P(dev["conics"]),
                                P(dev["colors"]), P(dev["opacities"]), P(dev["backgrounds"]),
                                None, P(dev["tile_offsets"]), P(dev["flatten_ids"]), P(rc),
                                P(ra), P(li), s) == 0
    assert_exact(to_np(li), e["last_ids"], "last_ids (length-ordered schedule)")
    assert_exact(to_np(ra), to_np(gs.rasterize_to_pixels_3dgs_forward(dev, W, H, ts)[
        "render_alphas"]), "alphas (length-ordered schedule)")
    # the cost record from the oracle's last ids
    off = inp["tile_offsets"].reshape(-1).astype(np.int64)
    end = np.append(off[1:], m)
    lp = np.full((th * ts, tw * ts), -1, np.int64)
    lp[:H, :W] = np.minimum(e["last_ids"][0], np.repeat(np.repeat(
        (end - 1).reshape(th, tw), ts, 0), ts, 1)[:H, :W])
    tmax = lp.reshape(th, ts, tw, ts).max(axis=(1, 3)).reshape(-1)
    want = np.maximum(0, tmax - off + 1)
    # a tile with a pixel whose stop decision was left to the fix-up pass
    # records its whole list
    got = to_np(cost).astype(np.int64)
    assert np.all((got == want) | (got == end - off)), "tile_cost"
    assert np.mean(got == want) > 0.95
    # the backward in the cost order equals the unordered backward
    assert lib.gs_raster_tile_order(ct.byref(rp), None, P(cost), P(order), s) == 0
    rng = np.random.default_rng(12)
    vrc = T(rng.normal(size=(1, H, W, 3)).astype(np.float32))
    vra = T(rng.normal(0, 0.1, size=(1, H, W, 1)).astype(np.float32))
    out = {k: torch.empty_like(dev[src]) for k, src in
           (("v_means2d", "means2d"), ("v_conics", "conics"), ("v_colors", "colors"),
            ("v_opacities", "opacities"), ("v_backgrounds", "backgrounds"))}
    assert lib.gs_rasterize_bwd(ct.byref(rp), P(dev["means2d"]), P(dev["conics"]),
                                P(dev["colors"]), P(dev["opacities"]), P(dev["backgrounds"]),
                                None, P(dev["tile_offsets"]), P(dev["flatten_ids"]), P(ra),
                                P(li), P(vrc), P(vra), None, P(out["v_means2d"]),
                                P(out["v_conics"]), P(out["v_colors"]), P(out["v_opacities"]),
                                P(out["v_backgrounds"]), s) == 0
    ref = gs.rasterize_to_pixels_3dgs_backward(dev, {"render_alphas": ra, "last_ids": li},
                                               {"v_render_colors": vrc, "v_render_alphas": vra},
                                               W, H, ts)
    for k, v in out.items():
        assert_grad_close(to_np(v), to_np(ref[k]), "ordered " + k, atol_frac=1e-5)


def test_rasterize_nonfinite_opacities(gs, oracle, golden, cuda):
    """NaN and infinite opacities decide as the reference does: its
    std::min(0.99f, NaN) is 0.99, so a NaN or +inf opacity is composited and
    clamped wherever sigma >= 0, and a -inf one exactly where its
    exponential underflows (-inf * 0 is NaN).  The oracle agrees with the
    reference's own eval_cpu on this case bit for bit."""
    d = golden("chain_cfg1")
    W, H, ts, inp = _raster_case(oracle, "chain_cfg1", d)
    op = inp["opacities"].copy()
    idx = np.random.default_rng(3).choice(op.size, 40, replace=False)
    op.reshape(-1)[idx[:15]] = np.nan
    op.reshape(-1)[idx[15:30]] = np.inf
    op.reshape(-1)[idx[30:]] = -np.inf
    inp["opacities"] = op
    e = oracle.raster_fwd(width=W, height=H, tile_size=ts, **inp)
    g = gs.rasterize_to_pixels_3dgs_forward({k: T(v) for k, v in inp.items()}, W, H, ts)
    assert_exact(to_np(g["last_ids"]), e["last_ids"], "last_ids")
    assert_fwd_close(to_np(g["render_alphas"]), e["render_alphas"], "alphas")
    assert_fwd_close(to_np(g["render_colors"]), e["render_colors"], "colors")
