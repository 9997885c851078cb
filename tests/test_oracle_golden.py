"""Pin the CPU oracle (oracle/gsplat_oracle.c) before trusting it.

1. Against tests/golden, produced by the reference's own eval_cpu code
   (tests/golden/make_golden.py): the restatement must agree bit for bit.
2. Against the known answers of the reference's C++ tests
   (gsplat_core/test/test.cpp), transcribed here as plain numbers.
3. Live against oracle/_ref when it was built in this checkout.
"""
from __future__ import annotations

import numpy as np
import pytest

from _util import assert_exact


def _chain_case(oracle, d):
    W, H, ts = int(d["width"]), int(d["height"]), int(d["tile_size"])
    tw, th = (W + ts - 1) // ts, (H + ts - 1) // ts
    out = {}
    proj = oracle.proj_fwd(d["means"][None], d["viewmats"][None], d["Ks"][None], W, H,
                           quats=d["quats"][None], scales=d["scales"][None],
                           opacities=d["opacities"][None], calc_compensations=True)
    out.update({"proj_" + k: v for k, v in proj.items()})
    m2 = proj["means2d"].reshape(1, -1, 2)
    rad = proj["radii"].reshape(1, -1, 2)
    dep = proj["depths"].reshape(1, -1)
    it = oracle.isect_tile(m2, rad, dep, 1, ts, tw, th, sort=True)
    iu = oracle.isect_tile(m2, rad, dep, 1, ts, tw, th, sort=False)
    out.update({"isect_" + k: v for k, v in it.items()})
    out.update({"isect_unsorted_" + k: v for k, v in iu.items()})
    out["tile_offsets"] = oracle.isect_offset(it["isect_ids"], 1, tw, th)
    deg = int(d["sh_degree"])
    out["sh_colors"] = oracle.sh_fwd(deg, d["dirs"], d["coeffs"])
    rf = oracle.raster_fwd(m2, proj["conics"].reshape(1, -1, 3), d["colors"],
                           d["opacities"][None], out["tile_offsets"], it["flatten_ids"], W, H, ts,
                           backgrounds=d["backgrounds"])
    out.update({"rf_" + k: v for k, v in rf.items()})
    rb = oracle.raster_bwd(m2, proj["conics"].reshape(1, -1, 3), d["colors"],
                           d["opacities"][None], out["tile_offsets"], it["flatten_ids"], W, H, ts,
                           rf["render_alphas"], rf["last_ids"], d["v_render_colors"],
                           d["v_render_alphas"], backgrounds=d["backgrounds"], absgrad=True,
                           threads=1)
    out.update({"rb_" + k: v for k, v in rb.items()})
    shb = oracle.sh_bwd(deg, d["dirs"], d["coeffs"], d["v_sh"])
    out.update({"shb_" + k: v for k, v in shb.items()})
    pb = oracle.proj_bwd(d["means"][None], d["viewmats"][None], d["Ks"][None], W, H,
                         proj["radii"], proj["conics"], d["v_means2d"], d["v_depths"],
                         d["v_conics"], quats=d["quats"][None], scales=d["scales"][None],
                         compensations=proj["compensations"], v_compensations=d["v_compensations"],
                         viewmats_requires_grad=True)
    out.update({"pb_" + k: v for k, v in pb.items()})
    return out


@pytest.mark.parametrize("name", ["chain_cfg1", "chain_cfg3"])
def test_oracle_matches_reference_chain(oracle, golden, name):
    d = golden(name)
    got = _chain_case(oracle, d)
    for k, v in got.items():
        assert k in d, k
        assert_exact(v, d[k], f"{name}:{k}")


def test_oracle_matches_reference_ops(oracle, golden):
    d = golden("ops")
    q, s = d["qs_quats"], d["qs_scales"]
    for triu in (0, 1):
        f = oracle.qs2c_fwd(q, s, True, True, bool(triu))
        assert_exact(f["covars"], d[f"qs_triu{triu}_covars"], "covars")
        assert_exact(f["precis"], d[f"qs_triu{triu}_precis"], "precis")
        b = oracle.qs2c_bwd(q, s, d[f"qs_triu{triu}_vc"], d[f"qs_triu{triu}_vp"], bool(triu))
        assert_exact(b["v_quats"], d[f"qs_triu{triu}_v_quats"], "v_quats")
        assert_exact(b["v_scales"], d[f"qs_triu{triu}_v_scales"], "v_scales")
    for deg in range(5):
        c = oracle.sh_fwd(deg, d["sh_dirs"], d["sh_coeffs"], d["sh_masks"])
        assert_exact(c, d[f"sh_deg{deg}_colors"], f"sh deg{deg}")
        b = oracle.sh_bwd(deg, d["sh_dirs"], d["sh_coeffs"], d["sh_vcol"], d["sh_masks"])
        assert_exact(b["v_dirs"], d[f"sh_deg{deg}_v_dirs"], f"sh v_dirs deg{deg}")
        assert_exact(b["v_coeffs"], d[f"sh_deg{deg}_v_coeffs"], f"sh v_coeffs deg{deg}")
    W, H = int(d["pc_width"]), int(d["pc_height"])
    p = oracle.proj_fwd(d["pc_means"], d["pc_viewmats"], d["pc_Ks"], W, H, covars=d["pc_covars"],
                        near_plane=2.4, far_plane=3.9)
    for k in ("means2d", "depths", "conics", "radii"):
        assert_exact(p[k], d["pc_" + k], "proj covars " + k)
    pb = oracle.proj_bwd(d["pc_means"], d["pc_viewmats"], d["pc_Ks"], W, H, p["radii"],
                         p["conics"], d["pc_vm2"], d["pc_vd"], d["pc_vco"], covars=d["pc_covars"],
                         viewmats_requires_grad=True)
    for k, v in pb.items():
        assert_exact(v, d["pcb_" + k], "proj bwd covars " + k)


# ----------------------------------------------------------------------------
# Known answers of gsplat_core/test/test.cpp

def test_known_intersect_dense_aabb(oracle):
    """test.cpp:653-737 and :739-855."""
    m2 = np.array([[[20, 20], [50, 50], [8, 8]]], np.float32)
    rad = np.array([[[10, 10], [5, 5], [0, 0]]], np.int32)
    dep = np.array([[1.0, 0.5, 2.0]], np.float32)
    r = oracle.isect_tile(m2, rad, dep, 1, 16, 4, 4, sort=True)
    assert r["tiles_per_gauss"].tolist() == [[4, 4, 0]]
    assert [(int(k) >> 32) & 0x1F for k in r["isect_ids"]] == [0, 1, 4, 5, 10, 11, 14, 15]
    assert r["flatten_ids"].tolist() == [0, 0, 0, 0, 1, 1, 1, 1]
    offs = oracle.isect_offset(r["isect_ids"], 1, 4, 4)
    assert offs.ravel().tolist() == [0, 1, 2, 2, 2, 3, 4, 4, 4, 4, 4, 5, 6, 6, 6, 7]
    u = oracle.isect_tile(m2, rad, dep, 1, 16, 4, 4, sort=False)
    exp = [(t << 32) | 0x3F800000 for t in (0, 1, 4, 5)] + [(t << 32) | 0x3F000000 for t in (10, 11, 14, 15)]
    assert u["isect_ids"].tolist() == exp


def test_known_intersect_prefix_sort(oracle):
    """test.cpp:857-1030: swapped Gaussians sort back into tile order."""
    m2 = np.array([[[50, 50], [20, 20], [8, 8]]], np.float32)
    rad = np.array([[[5, 5], [10, 10], [0, 0]]], np.int32)
    dep = np.array([[0.5, 1.0, 2.0]], np.float32)
    u = oracle.isect_tile(m2, rad, dep, 1, 16, 4, 4, sort=False)
    s = oracle.isect_tile(m2, rad, dep, 1, 16, 4, 4, sort=True)
    assert u["isect_ids"].tolist() == [(t << 32) | 0x3F000000 for t in (10, 11, 14, 15)] + \
        [(t << 32) | 0x3F800000 for t in (0, 1, 4, 5)]
    assert s["isect_ids"].tolist() == [(t << 32) | 0x3F800000 for t in (0, 1, 4, 5)] + \
        [(t << 32) | 0x3F000000 for t in (10, 11, 14, 15)]
    assert s["flatten_ids"].tolist() == [1, 1, 1, 1, 0, 0, 0, 0]


def test_known_rasterize_closed_form(oracle):
    """test.cpp:1067-1134 (one Gaussian, 2x2 image) and :1199-1271 (masks)."""
    kw = dict(means2d=np.array([[[1.0, 1.0]]], np.float32),
              conics=np.array([[[1.0, 0.0, 1.0]]], np.float32),
              colors=np.array([[[1.0, 0.0, 0.0]]], np.float32),
              opacities=np.array([[0.5]], np.float32),
              flatten_ids=np.array([0], np.int32), tile_size=2,
              backgrounds=np.array([[0.1, 0.2, 0.3]], np.float32))
    r = oracle.raster_fwd(tile_offsets=np.zeros((1, 1, 1), np.int32), width=2, height=2, **kw)
    a = 0.5 * np.exp(-0.25)
    Tt = 1 - a
    assert np.allclose(r["render_alphas"].ravel(), a, atol=1e-5)
    assert np.allclose(r["render_colors"].reshape(4, 3), [a + Tt * 0.1, Tt * 0.2, Tt * 0.3], atol=1e-5)
    assert r["last_ids"].ravel().tolist() == [0, 0, 0, 0]
    rm = oracle.raster_fwd(tile_offsets=np.array([[[0, 1]]], np.int32), width=4, height=2,
                           masks=np.array([[[True, False]]]), **kw)
    alphas = rm["render_alphas"].reshape(2, 4)
    assert np.allclose(alphas[:, :2], a, atol=1e-5) and np.allclose(alphas[:, 2:], 0.0)
    assert np.allclose(rm["render_colors"].reshape(2, 4, 3)[:, 2:], [0.1, 0.2, 0.3], atol=1e-6)


def test_known_sh_closed_form(oracle):
    """test.cpp:1388-1460 (degree 0/1, masks) and :1563-1623 (backward)."""
    c0, c1 = 0.2820947917738781, 0.48860251190292
    dirs = np.array([[0, 0, 1], [1, 0, 0]], np.float32)
    co = np.array([[1, 2, 3], [.1, .2, .3], [.4, .5, .6], [.7, .8, .9],
                   [4, 5, 6], [0, 0, 0], [0, 0, 0], [0, 0, 0]], np.float32).reshape(2, 4, 3)
    d0 = oracle.sh_fwd(0, dirs, co)
    assert np.allclose(d0[0], [c0 * 1, c0 * 2, c0 * 3], atol=1e-6)
    d1 = oracle.sh_fwd(1, dirs, co)
    assert np.allclose(d1[0], [c0 + c1 * .4, 2 * c0 + c1 * .5, 3 * c0 + c1 * .6], atol=1e-6)
    assert np.allclose(d1[1], [c0 * 4, c0 * 5, c0 * 6], atol=1e-6)
    dm = oracle.sh_fwd(0, dirs, co, masks=np.array([True, False]))
    assert np.allclose(dm[1], 0.0)
    b = oracle.sh_bwd(1, dirs[:1], co[:1], np.array([[1, 2, 3]], np.float32))
    assert np.allclose(b["v_coeffs"][0, 0], [c0, 2 * c0, 3 * c0], atol=1e-6)
    assert np.allclose(b["v_coeffs"][0, 2], [c1, 2 * c1, 3 * c1], atol=1e-6)
    assert np.allclose(b["v_dirs"][0], [-c1 * 5.0, -c1 * 1.4, 0.0], atol=5e-4)


def test_known_quat_scale_closed_form(oracle):
    """test.cpp:1690-1760 and :1878-1954."""
    q = np.array([[1, 0, 0, 0], [2, 0, 0, 0]], np.float32)
    s = np.array([[2, 3, 4], [0.5, 2, 4]], np.float32)
    r = oracle.qs2c_fwd(q, s)
    assert np.allclose(r["covars"], [[4, 0, 0, 9, 0, 16], [0.25, 0, 0, 4, 0, 16]], atol=1e-6)
    assert np.allclose(r["precis"], [[.25, 0, 0, 1 / 9, 0, 1 / 16], [4, 0, 0, .25, 0, 1 / 16]], atol=1e-6)
    q2 = np.array([[1, 0, 0, 0], [0.9238795, 0.3826834, 0, 0]], np.float32)
    s2 = np.array([[2, 3, 4], [0.5, 1.5, 2.5]], np.float32)
    vc = np.array([[.1, 0, 0, .2, 0, .3], [-.2, .05, .1, .4, -.15, .25]], np.float32)
    vp = np.array([[.4, 0, 0, .5, 0, .6], [.3, -.25, .35, -.1, .2, .45]], np.float32)
    b = oracle.qs2c_bwd(q2, s2, vc, vp)
    assert np.allclose(b["v_scales"][0], [0.3, 1.2 - 1 / 27, 2.4 - 0.01875], atol=3e-3)
    assert np.allclose(b["v_quats"][0], 0.0, atol=3e-3)


def test_known_projection_pinhole(oracle):
    """test.cpp:60-130 analytic pinhole reference and :261-350."""
    W = H = 64
    fx = fy = 50.0
    cx = cy = 32.0
    means = np.array([[[0, 0, 1], [0.25, -0.25, 2]]], np.float32)
    quats = np.array([[[1, 0, 0, 0], [1, 0, 0, 0]]], np.float32)
    scales = np.array([[[.1, .1, .1], [.2, .2, .2]]], np.float32)
    view = np.eye(4, dtype=np.float32)[None, None]
    K = np.array([[[[fx, 0, cx], [0, fy, cy], [0, 0, 1]]]], np.float32)
    r = oracle.proj_fwd(means, view, K, W, H, quats=quats, scales=scales,
                        opacities=np.array([[0.8, 0.6]], np.float32), calc_compensations=True,
                        far_plane=100.0)
    for i, (x, y, z, var, op) in enumerate([(0, 0, 1, .01, .8), (.25, -.25, 2, .04, .6)]):
        tfx, tfy = 0.5 * W / fx, 0.5 * H / fy
        lxp, lxn = (W - cx) / fx + 0.3 * tfx, cx / fx + 0.3 * tfx
        lyp, lyn = (H - cy) / fy + 0.3 * tfy, cy / fy + 0.3 * tfy
        rz = 1 / z
        tx, ty = z * min(lxp, max(-lxn, x * rz)), z * min(lyp, max(-lyn, y * rz))
        j00, j02, j11, j12 = fx * rz, -fx * tx * rz * rz, fy * rz, -fy * ty * rz * rz
        c00, c01, c11 = var * (j00 ** 2 + j02 ** 2), var * j02 * j12, var * (j11 ** 2 + j12 ** 2)
        det_o = c00 * c11 - c01 ** 2
        c00 += 0.3
        c11 += 0.3
        det = c00 * c11 - c01 ** 2
        comp = np.sqrt(max(0.005 ** 2, det_o / det))
        ext = min(3.33, np.sqrt(2 * np.log(op * comp * 255)))
        assert r["radii"][0, 0, i].tolist() == [int(np.ceil(ext * np.sqrt(c00))), int(np.ceil(ext * np.sqrt(c11)))]
        assert np.allclose(r["means2d"][0, 0, i], [fx * x * rz + cx, fy * y * rz + cy], atol=1e-4)
        assert np.allclose(r["conics"][0, 0, i], [c11 / det, -c01 / det, c00 / det], atol=1e-4)
        assert np.allclose(r["compensations"][0, 0, i], comp, atol=1e-4)


def test_known_projection_culling(oracle):
    """test.cpp:352-437: near, far and radius_clip culling."""
    means = np.array([[[0, 0, 1], [0, 0, 0.001], [0, 0, 200], [0.25, -0.25, 2]]], np.float32)
    quats = np.tile(np.array([1, 0, 0, 0], np.float32), (1, 4, 1))
    scales = np.array([[[.1] * 3, [.1] * 3, [.1] * 3, [.001] * 3]], np.float32)
    view = np.eye(4, dtype=np.float32)[None, None]
    K = np.array([[[[50, 0, 32], [0, 50, 32], [0, 0, 1]]]], np.float32)
    r = oracle.proj_fwd(means, view, K, 64, 64, quats=quats, scales=scales, far_plane=100.0,
                        radius_clip=2.0)
    rad = r["radii"][0, 0]
    assert rad[0, 0] > 2 and rad[0, 1] > 2
    assert (rad[1:] == 0).all()
    assert r["compensations"].shape == (0,)


def test_oracle_against_live_reference(oracle):
    """When oracle/_ref was built here, cross-check a fresh random case."""
    from oracle.oracle import Reference
    if not Reference.available():
        pytest.skip("oracle/_ref not built in this checkout")
    ref = Reference()
    rng = np.random.default_rng(123)
    dirs = rng.normal(size=(500, 3)).astype(np.float32)
    co = rng.normal(size=(500, 16, 3)).astype(np.float32)
    assert_exact(oracle.sh_fwd(3, dirs, co), ref.sh_fwd(3, dirs, co), "sh live")
    ids = np.sort(rng.integers(0, 1 << 45, size=5000)).astype(np.int64)
    assert_exact(oracle.isect_offset(ids, 2, 64, 64), ref.isect_offset(ids, 2, 64, 64), "offsets")


def test_oracle_nonfinite_opacities_match_reference(oracle, golden):
    """NaN / +inf / -inf opacities: the oracle's rasterizer forward decides
    as the reference's eval_cpu (std::min(0.99f, NaN) is 0.99)."""
    from oracle.oracle import Reference
    if not Reference.available():
        pytest.skip("oracle/_ref not built in this checkout")
    ref = Reference()
    d = golden("chain_cfg1")
    W, H, ts = int(d["width"]), int(d["height"]), int(d["tile_size"])
    op = d["opacities"].copy()
    idx = np.random.default_rng(3).choice(op.size, 40, replace=False)
    op[idx[:15]], op[idx[15:30]], op[idx[30:]] = np.nan, np.inf, -np.inf
    inp = dict(means2d=d["proj_means2d"].reshape(1, -1, 2),
               conics=d["proj_conics"].reshape(1, -1, 3), colors=d["colors"],
               opacities=op[None], tile_offsets=d["tile_offsets"],
               flatten_ids=d["isect_flatten_ids"])
    a = oracle.raster_fwd(width=W, height=H, tile_size=ts, threads=1, **inp)
    b = ref.raster_fwd(width=W, height=H, tile_size=ts, **inp)
    for k in a:
        assert_exact(a[k], b[k], "non-finite opacities " + k)


def _densify_cfg(d):
    cfg = {k: float(d[k]) for k in ("grow_grad2d", "grow_scale3d", "grow_scale2d", "prune_opa",
                                    "prune_scale3d", "prune_scale2d", "scene_scale")}
    cfg["refine_scale2d_stop_iter"] = int(d["refine_scale2d_stop_iter"])
    cfg["reset_every"] = int(d["reset_every"])
    return cfg


def test_densify_oracle_matches_reference(golden):
    """oracle/densify.py against the reference trainer's own
    ScannerDefaultStrategyRuntime (tests/golden/make_densify_golden.py):
    statistics bit for bit, clone selection, split mask, prune keep set."""
    from oracle import densify as D
    d = golden("densify")
    n = int(d["N"])
    g, c, r = (np.zeros(n, np.float32) for _ in range(3))
    for t in range(d["v_means2d"].shape[0]):
        D.accumulate(d["v_means2d"][t], d["radii_in"][t], int(d["W"]), int(d["H"]), int(d["C"]),
                     g, c, r)
    assert_exact(g, d["grad2d"], "grad2d")
    assert_exact(c, d["count"], "count")
    assert_exact(r, d["radii"], "radii")
    cfg = _densify_cfg(d)
    m = D.masks(g, c, r, d["log_scales"], d["opacity_logits"], int(d["step"]), n, cfg,
                grow=True, prune=False)
    assert_exact(np.nonzero(m["clone"])[0], d["clone_selected"], "clone selection")
    assert_exact(m["split"], d["split_mask"][:n], "split mask")
    assert not d["split_mask"][n:].any()
    p = D.masks(None, None, d["prune_radii"], d["prune_log_scales"], d["prune_opacity_logits"],
                int(d["step"]), n, cfg, grow=False, prune=True)
    assert_exact(np.nonzero(~p["prune"])[0], d["prune_keep"], "prune keep set")
    assert_exact(p["prune_breakdown"], d["prune_breakdown"], "prune breakdown")


def test_parallel_reference_step_matches_one_thread(oracle):
    """bench.py's reference arm splits the reference's step over host
    threads (oracle/ref_step.py): Gaussian chunks, a stable merge of the
    chunks' sorted lists, tile sets per thread.  Its lists and forward
    outputs are those of one single-threaded pass bit for bit, its
    gradients the same up to the order of the float sums."""
    from gsplat_core import synthetic as S
    from oracle.ref_step import ParallelReferenceStep, metal_cull
    sc = S.config3(seed=3, n=20_000)
    sc.Ks = sc.Ks.copy()
    sc.Ks[:, :2, :] /= 4
    sc.width, sc.height = sc.width // 4, sc.height // 4
    vrc, vra = S.cotangents(3, 1, sc.height, sc.width)
    st = ParallelReferenceStep(oracle, sc, vrc, vra, threads=5)
    _, m, _ = st.run()
    st.close()
    got = st.last
    W, H = sc.width, sc.height
    p = metal_cull(oracle.proj_fwd(sc.means[None], sc.viewmats[None], sc.Ks[None], W, H,
                                   quats=sc.quats[None], scales=sc.scales[None]), W, H)
    N = sc.n
    it = oracle.isect_tile(p["means2d"].reshape(1, N, 2), p["radii"].reshape(1, N, 2),
                           p["depths"].reshape(1, N), 1, 16, sc.tile_width, sc.tile_height)
    assert m == it["isect_ids"].size
    assert_exact(got["isect_ids"], it["isect_ids"], "keys")
    assert_exact(got["flatten_ids"], it["flatten_ids"], "flatten ids")
    offs = oracle.isect_offset(it["isect_ids"], 1, sc.tile_width, sc.tile_height)
    assert_exact(got["tile_offsets"], offs, "offsets")
    kw = dict(means2d=p["means2d"].reshape(1, N, 2), conics=p["conics"].reshape(1, N, 3),
              colors=got["colors"], opacities=sc.opacities[None], tile_offsets=offs,
              flatten_ids=it["flatten_ids"], width=W, height=H, tile_size=16)
    rf = oracle.raster_fwd(threads=1, **kw)
    for k, v in rf.items():
        assert_exact(got["rf_" + k], v, k)
    rb = oracle.raster_bwd(render_alphas=rf["render_alphas"], last_ids=rf["last_ids"],
                           v_render_colors=vrc, v_render_alphas=vra, threads=1, **kw)
    for k, v in rb.items():
        scale = np.abs(v).max()
        assert np.allclose(got["rb_" + k], v, rtol=1e-4, atol=1e-5 * scale), k
