"""Host logic of the camera-sharded step (gsplat_core.sharded) on CPU:
camera slicing, exchange choice, and both gradient exchanges run by two
gloo ranks, each over the oracle's gradients of its own cameras, against the
oracle's single-process step over all cameras."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from _util import assert_grad_close


def test_camera_shard_covers_every_camera_once():
    from gsplat_core.sharded import camera_shard
    for C in range(0, 40):
        for w in range(1, 9):
            got = [camera_shard(C, w, r) for r in range(w)]
            assert got[0][0] == 0 and got[-1][1] == C
            for (a, b), (c, _) in zip(got[:-1], got[1:]):
                assert b == c
            sizes = [b - a for a, b in got]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        camera_shard(4, 2, 2)


def test_exchange_choice():
    from gsplat_core.sharded import choose_exchange, exchange_bytes
    n = 1_000_000
    assert choose_exchange(n, 16, 1, 1) == "allreduce"
    assert choose_exchange(n, 16, 1, 8) == "gather"         # one camera per rank
    assert choose_exchange(n, 16, 1, 2) == "gather"
    assert choose_exchange(n, 16, 4, 8) == "shard"          # 32 cameras on 8 GPUs
    assert choose_exchange(n + 1, 16, 1, 8) == "gather"     # uneven slices
    assert choose_exchange(n + 1, 16, 3, 8) == "gather"
    assert choose_exchange(n + 1, 16, 4, 8) == "allreduce"
    assert choose_exchange(n, 1, 1, 8) == "allreduce"       # SH degree 0
    # shard moves fewer bytes than the all-reduce for the 32-camera batch
    assert exchange_bytes("shard", n, 16, 4, 8) < exchange_bytes("allreduce", n, 16, 4, 8)
    assert exchange_bytes("allreduce", n, 16, 1, 2) == pytest.approx(236e6)


def _scene():
    from gsplat_core import synthetic as S
    sc = S.config3(seed=3, n=60_000)
    C = 4
    sc.viewmats = S.orbit(C, 4.0)
    sc.Ks = np.repeat(sc.Ks[:1], C, 0).copy()
    sc.Ks[:, :2, :] /= 8
    sc.width, sc.height = sc.width // 8, sc.height // 8
    idx = np.sort(np.random.default_rng(1).choice(sc.n, size=3000, replace=False))
    for k in ("means", "quats", "scales", "opacities", "coeffs"):
        setattr(sc, k, getattr(sc, k)[idx])
    vrc, vra = S.cotangents(5, C, sc.height, sc.width)
    return sc, vrc, vra


def _camera_grads(oracle, sc, cams, vrc, vra, with_sh):
    """The oracle's step for cameras ``cams``: projection part of the
    gradients, colour cotangents, and (with_sh) the SH glue backward."""
    W, H, ts, tw, th = sc.width, sc.height, sc.tile_size, sc.tile_width, sc.tile_height
    C = len(cams)
    view, Ks = sc.viewmats[cams], sc.Ks[cams]
    p = oracle.proj_fwd(sc.means[None], view[None], Ks[None], W, H, quats=sc.quats[None],
                        scales=sc.scales[None])
    vis = (p["radii"][0, ..., 0] > 0) & (p["radii"][0, ..., 1] > 0)
    colors = oracle.sh_glue_fwd(sc.sh_degree, sc.means, view, sc.coeffs, vis)
    m2 = p["means2d"].reshape(C, -1, 2)
    it = oracle.isect_tile(m2, p["radii"].reshape(C, -1, 2), p["depths"].reshape(C, -1), C, ts,
                           tw, th)
    offs = oracle.isect_offset(it["isect_ids"], C, tw, th)
    op = np.broadcast_to(sc.opacities, (C, sc.n)).copy()
    kw = dict(means2d=m2, conics=p["conics"].reshape(C, -1, 3), colors=colors, opacities=op,
              tile_offsets=offs, flatten_ids=it["flatten_ids"], width=W, height=H, tile_size=ts,
              backgrounds=np.zeros((C, 3), np.float32))
    rf = oracle.raster_fwd(**kw)
    rb = oracle.raster_bwd(render_alphas=rf["render_alphas"], last_ids=rf["last_ids"],
                           v_render_colors=vrc[cams], v_render_alphas=vra[cams], **kw)
    pb = oracle.proj_bwd(sc.means[None], view[None], Ks[None], W, H, p["radii"], p["conics"],
                         rb["v_means2d"][None], np.zeros(p["depths"].shape, np.float32),
                         rb["v_conics"][None], quats=sc.quats[None], scales=sc.scales[None])
    v_means = pb["v_means"][0].copy()
    v_coeffs = np.zeros_like(sc.coeffs)
    if with_sh:
        gb = oracle.sh_glue_bwd(sc.sh_degree, sc.means, view, sc.coeffs, rb["v_colors"], vis)
        v_means += gb["v_means"]
        v_coeffs = gb["v_coeffs"]
    flat = np.concatenate([v_means.ravel(), pb["v_quats"][0].ravel(), pb["v_scales"][0].ravel(),
                           rb["v_opacities"].sum(0).ravel(), v_coeffs.ravel()])
    return flat.astype(np.float32), rb["v_colors"]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle.oracle import Oracle
        from gsplat_core.sharded import _all_gather, camera_shard, exchange_gradients
        oracle = Oracle()
        sc, vrc, vra = _scene()
        a, b = camera_shard(sc.viewmats.shape[0], world, rank)
        cams = list(range(a, b))
        flat_np, v_colors = _camera_grads(oracle, sc, cams, vrc, vra, with_sh=(mode == "allreduce"))
        if mode == "shard":
            flat_np[11 * sc.n:] = 0.0
        v_local = torch.from_numpy(np.ascontiguousarray(v_colors))
        flat = torch.from_numpy(flat_np)
        v_all = torch.empty((sc.viewmats.shape[0], sc.n, 3), dtype=torch.float32)
        n, K = sc.n, sc.coeffs.shape[1]

        def sh_backward(v_colors_all):
            gb = oracle.sh_glue_bwd(sc.sh_degree, sc.means, sc.viewmats, sc.coeffs,
                                    v_colors_all.numpy(), None)
            flat[11 * n:] = torch.from_numpy(gb["v_coeffs"].ravel())
            return torch.from_numpy(gb["v_means"])

        if mode == "shard":
            from gsplat_core.sharded import PROJ_FIELDS, shard_exchange, start_shard_all_to_all
            ns = n // world
            C_local = len(cams)
            recv = torch.empty((sc.viewmats.shape[0], ns, 3), dtype=torch.float32)
            reduced = [torch.empty(d * ns, dtype=torch.float32) for _, d in PROJ_FIELDS]
            coeff_slice = torch.empty((ns, K, 3), dtype=torch.float32)
            moving = start_shard_all_to_all(recv, v_local, None)
            # recv row j * world + g holds camera j of rank g
            perm = [g * C_local + j for j in range(C_local) for g in range(world)]
            a = rank * ns

            def sh_slice():
                gb = oracle.sh_glue_bwd(sc.sh_degree, sc.means[a:a + ns], sc.viewmats[perm],
                                        sc.coeffs[a:a + ns], recv.numpy(), None)
                coeff_slice.copy_(torch.from_numpy(gb["v_coeffs"]))
                reduced[0].add_(torch.from_numpy(gb["v_means"]).reshape(-1))

            shard_exchange(flat, n, K, reduced, coeff_slice, sh_slice, moving)
            np.save(os.path.join(out_dir, f"{mode}_{rank}.npy"), flat.numpy())
            return
        gathering = None
        if mode == "gather_started":
            # the sharded step starts the colour all-gather before its
            # projection backward and hands the handle over
            gathering = _all_gather(v_all.view(-1), v_local.reshape(-1), None, async_op=True)
        exchange_gradients("gather" if mode == "gather_started" else mode, flat, n, v_local, v_all,
                           sh_backward, gathering=gathering)
        np.save(os.path.join(out_dir, f"{mode}_{rank}.npy"), flat.numpy())
        assert K == 16
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["allreduce", "gather", "gather_started", "shard"])
def test_two_rank_exchange_matches_single_process(oracle, tmp_path, mode):
    sc, vrc, vra = _scene()
    expect, _ = _camera_grads(oracle, sc, list(range(sc.viewmats.shape[0])), vrc, vra, True)
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
        if p.is_alive():
            p.kill()
            pytest.fail(f"rank {p.name} did not finish")
        assert p.exitcode == 0
    outs = [np.load(tmp_path / f"{mode}_{r}.npy") for r in range(2)]
    np.testing.assert_array_equal(outs[0], outs[1])   # every rank holds the same sums
    n = sc.n
    names = (("v_means", 0, 3 * n), ("v_quats", 3 * n, 7 * n), ("v_scales", 7 * n, 10 * n),
             ("v_opacities", 10 * n, 11 * n), ("v_coeffs", 11 * n, outs[0].size))
    for name, a, b in names:
        assert_grad_close(outs[0][a:b], expect[a:b], f"{mode} {name}", atol_frac=1e-5)
    assert np.abs(expect[11 * n:]).max() > 0
