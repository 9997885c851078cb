"""Generate the golden fixtures of tests/golden from the reference itself.

Runs the reference's own eval_cpu code (gsplat_core/*.cpp compiled in place
against oracle/mlx_shim by `make -C oracle ref`, loaded through
oracle/oracle.py:Reference) on small seeded inputs and on the known-answer
inputs of gsplat_core/test/test.cpp, and stores inputs and outputs as .npz.
The projection forward outputs get the Metal eval_gpu culling applied
(metal/gsplat_projection.metal:314-326) after the fact -- the reference's
CPU path skips it -- without changing the reference code.

    make -C oracle ref && python tests/golden/make_golden.py
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "gsplat-mlx_b200"))

from oracle.oracle import Reference  # noqa: E402
from gsplat_core import synthetic as S  # noqa: E402


def metal_cull(out, width, height):
    m2, rad = out["means2d"], out["radii"]
    off = ((m2[..., 0] + rad[..., 0] <= 0) | (m2[..., 0] - rad[..., 0] >= width) |
           (m2[..., 1] + rad[..., 1] <= 0) | (m2[..., 1] - rad[..., 1] >= height))
    for k in ("means2d", "conics", "radii"):
        out[k][off] = 0
    out["depths"][off] = 0
    if out["compensations"].size:
        out["compensations"][off] = 0
    return out


def save(name, **arrays):
    path = os.path.join(HERE, name + ".npz")
    np.savez_compressed(path, **arrays)
    print(f"wrote {path} ({os.path.getsize(path)} bytes)")


def chain(ref, scene, n_keep, seed):
    """Projection -> intersect -> offsets -> SH -> rasterize fwd/bwd ->
    projection bwd on a small seeded subset of a benchmark scene."""
    rng = np.random.default_rng(seed)
    idx = np.sort(rng.choice(scene.n, size=n_keep, replace=False))
    means, quats, scales = scene.means[idx], scene.quats[idx], scene.scales[idx]
    opac, coeffs = scene.opacities[idx], scene.coeffs[idx]
    W, H, ts = scene.width, scene.height, scene.tile_size
    tw, th = scene.tile_width, scene.tile_height
    view, K = scene.viewmats[:1], scene.Ks[:1]
    proj = metal_cull(ref.proj_fwd(means[None], view[None], K[None], W, H, quats=quats[None],
                                   scales=scales[None], opacities=opac[None],
                                   calc_compensations=True), W, H)
    m2 = proj["means2d"].reshape(1, -1, 2)
    rad = proj["radii"].reshape(1, -1, 2)
    dep = proj["depths"].reshape(1, -1)
    it = ref.isect_tile(m2, rad, dep, 1, ts, tw, th, sort=True)
    iu = ref.isect_tile(m2, rad, dep, 1, ts, tw, th, sort=False)
    offs = ref.isect_offset(it["isect_ids"], 1, tw, th)
    campos = -(view[0, :3, :3].T @ view[0, :3, 3])
    dirs = (means - campos).astype(np.float32)
    deg = scene.sh_degree
    sh = ref.sh_fwd(deg, dirs, coeffs)
    colors = np.clip(sh + 0.5, 0.0, 1.0).astype(np.float32)[None]
    bg = np.array([[0.1, 0.2, 0.3]], np.float32)
    con = proj["conics"].reshape(1, -1, 3)
    op = opac[None]
    rf = ref.raster_fwd(m2, con, colors, op, offs, it["flatten_ids"], W, H, ts, backgrounds=bg)
    vrc, vra = S.cotangents(seed, 1, H, W)
    rb = ref.raster_bwd(m2, con, colors, op, offs, it["flatten_ids"], W, H, ts,
                        rf["render_alphas"], rf["last_ids"], vrc, vra, backgrounds=bg,
                        absgrad=True)
    v_sh = rng.normal(size=dirs.shape).astype(np.float32)
    shb = ref.sh_bwd(deg, dirs, coeffs, v_sh)
    vm2 = rng.normal(size=proj["means2d"].shape).astype(np.float32)
    vd = rng.normal(size=proj["depths"].shape).astype(np.float32)
    vco = rng.normal(size=proj["conics"].shape).astype(np.float32)
    vcp = rng.normal(size=proj["depths"].shape).astype(np.float32)
    pb = ref.proj_bwd(means[None], view[None], K[None], W, H, proj["radii"], proj["conics"],
                      vm2, vd, vco, quats=quats[None], scales=scales[None],
                      compensations=proj["compensations"], v_compensations=vcp,
                      viewmats_requires_grad=True)
    out = dict(means=means, quats=quats, scales=scales, opacities=opac, coeffs=coeffs,
               viewmats=view, Ks=K, width=W, height=H, tile_size=ts, sh_degree=deg,
               backgrounds=bg, dirs=dirs, v_sh=v_sh, v_render_colors=vrc, v_render_alphas=vra,
               v_means2d=vm2, v_depths=vd, v_conics=vco, v_compensations=vcp, colors=colors)
    out.update({"proj_" + k: v for k, v in proj.items()})
    out.update({"isect_" + k: v for k, v in it.items()})
    out.update({"isect_unsorted_" + k: v for k, v in iu.items()})
    out["tile_offsets"] = offs
    out["sh_colors"] = sh
    out.update({"rf_" + k: v for k, v in rf.items()})
    out.update({"rb_" + k: v for k, v in rb.items()})
    out.update({"shb_" + k: v for k, v in shb.items()})
    out.update({"pb_" + k: v for k, v in pb.items()})
    return out


def ops(ref, seed=1):
    """Per-op cases that the chain does not exercise."""
    rng = np.random.default_rng(seed)
    out = {}
    n = 257
    q = rng.normal(size=(n, 4)).astype(np.float32)
    s = np.exp(rng.uniform(-2, 1, size=(n, 3))).astype(np.float32)
    for triu in (0, 1):
        f = ref.qs2c_fwd(q, s, True, True, bool(triu))
        shape = (n, 6) if triu else (n, 3, 3)
        vc = rng.normal(size=shape).astype(np.float32)
        vp = rng.normal(size=shape).astype(np.float32)
        b = ref.qs2c_bwd(q, s, vc, vp, bool(triu))
        out[f"qs_triu{triu}_covars"], out[f"qs_triu{triu}_precis"] = f["covars"], f["precis"]
        out[f"qs_triu{triu}_vc"], out[f"qs_triu{triu}_vp"] = vc, vp
        out[f"qs_triu{triu}_v_quats"], out[f"qs_triu{triu}_v_scales"] = b["v_quats"], b["v_scales"]
    out["qs_quats"], out["qs_scales"] = q, s
    # SH: every degree 0..4 with K = 25 rows, masks, one zero direction.
    m = 129
    dirs = rng.normal(size=(m, 3)).astype(np.float32)
    dirs[5] = 0.0
    co = rng.normal(size=(m, 25, 3)).astype(np.float32)
    masks = rng.uniform(size=m) > 0.2
    vcol = rng.normal(size=(m, 3)).astype(np.float32)
    out["sh_dirs"], out["sh_coeffs"], out["sh_masks"], out["sh_vcol"] = dirs, co, masks, vcol
    for d in range(5):
        out[f"sh_deg{d}_colors"] = ref.sh_fwd(d, dirs, co, masks)
        b = ref.sh_bwd(d, dirs, co, vcol, masks)
        out[f"sh_deg{d}_v_dirs"], out[f"sh_deg{d}_v_coeffs"] = b["v_dirs"], b["v_coeffs"]
    # Projection with covariances, two cameras, near/far culling, 2 batches.
    B, C, N = 2, 2, 300
    means = rng.uniform(-1, 1, size=(B, N, 3)).astype(np.float32)
    means[..., 2] *= 3
    A = rng.normal(size=(B, N, 3, 3)) * 0.05
    cov = A @ np.swapaxes(A, -1, -2) + np.eye(3) * 1e-3
    covars = np.stack([cov[..., 0, 0], cov[..., 0, 1], cov[..., 0, 2], cov[..., 1, 1],
                       cov[..., 1, 2], cov[..., 2, 2]], -1).astype(np.float32)
    views = np.stack([np.stack([S.look_at((0.3 * c, -0.2, -3.0 - b)) for c in range(C)])
                      for b in range(B)]).astype(np.float32)
    Ks = np.broadcast_to(S.intrinsics(80, 80, 40, 30), (B, C, 3, 3)).astype(np.float32).copy()
    W, H = 80, 60
    p = metal_cull(ref.proj_fwd(means, views, Ks, W, H, covars=covars, near_plane=2.4,
                                far_plane=3.9), W, H)
    out.update({"pc_means": means, "pc_covars": covars, "pc_viewmats": views, "pc_Ks": Ks,
                "pc_width": W, "pc_height": H})
    out.update({"pc_" + k: v for k, v in p.items()})
    vm2 = rng.normal(size=p["means2d"].shape).astype(np.float32)
    vd = rng.normal(size=p["depths"].shape).astype(np.float32)
    vco = rng.normal(size=p["conics"].shape).astype(np.float32)
    pb = ref.proj_bwd(means, views, Ks, W, H, p["radii"], p["conics"], vm2, vd, vco,
                      covars=covars, viewmats_requires_grad=True)
    out.update({"pc_vm2": vm2, "pc_vd": vd, "pc_vco": vco})
    out.update({"pcb_" + k: v for k, v in pb.items()})
    return out


def downscale(scene, factor):
    """The same scene seen by the same camera at 1/factor resolution."""
    import dataclasses
    K = scene.Ks.copy()
    K[:, :2, :] /= factor
    return dataclasses.replace(scene, Ks=K, width=scene.width // factor,
                               height=scene.height // factor)


def main():
    if not Reference.available():
        raise SystemExit("build the reference first: make -C oracle ref")
    ref = Reference()
    save("chain_cfg1", **chain(ref, S.config1(seed=0), 2000, seed=11))
    save("chain_cfg3", **chain(ref, downscale(S.config3(seed=0, n=200_000), 4), 6000, seed=12))
    save("ops", **ops(ref))


if __name__ == "__main__":
    main()
