"""The reference's CPU training step on every host thread (TEST / BENCHMARK
INFRASTRUCTURE ONLY: bench.py's reference arm and CPU baseline use it; the
product never does).

One step is what the reference trainer runs per camera (scripts/test/
scanner_points_training_utils.py:2076-2119): projection forward, the SH
colour glue, intersect (count, scan, encode, stable key sort), tile offsets,
rasterize forward and backward, SH backward, projection backward -- every
operator through the reference's own eval_cpu code (``Reference``, the
shim-compiled gsplat_core sources) or the C restatement (``Oracle``).

The eval_cpu bodies are serial loops; this driver splits the work across
host threads without changing any operator's arithmetic:

* per-Gaussian operators (projection, SH, their backward passes) run on
  contiguous Gaussian chunks, one call per chunk;
* the intersect pipeline runs per Gaussian chunk (count, scan and encode of
  the chunk, and its stable sort); the chunks' sorted lists are merged by a
  stable sort of their concatenation, which keeps equal keys in Gaussian
  order -- the order of one stable sort of the whole encode;
* the rasterizer runs once per thread with a tile mask (tiles dealt out
  round-robin); the forward outputs are taken from the owning thread, the
  backward gradients summed over threads.

The projection outputs get the Metal eval_gpu culling (footprints entirely
off the image, gsplat_core/metal/gsplat_projection.metal:319-326), which the
Python binding's path applies and the CPU path does not, so that the step
lists the same intersections as the GPU step.
"""
from __future__ import annotations

import os
import time
from concurrent.futures import ThreadPoolExecutor

import numpy as np


def host_threads() -> int:
    return max(1, len(os.sched_getaffinity(0)))


def metal_cull(out, width, height):
    """Zero the projection outputs of footprints entirely off the image
    (metal/gsplat_projection.metal:319-326)."""
    m2, rad = out["means2d"], out["radii"]
    off = ((m2[..., 0] + rad[..., 0] <= 0) | (m2[..., 0] - rad[..., 0] >= width) |
           (m2[..., 1] + rad[..., 1] <= 0) | (m2[..., 1] - rad[..., 1] >= height))
    for k in ("means2d", "conics", "radii"):
        out[k][off] = 0
    out["depths"][off] = 0
    if out["compensations"].size:
        out["compensations"][off] = 0
    return out


def _chunks(n, parts):
    edges = np.linspace(0, n, parts + 1).astype(np.int64)
    return [(int(a), int(b)) for a, b in zip(edges[:-1], edges[1:]) if b > a]


class ParallelReferenceStep:
    """One camera's training step of a scene (``sc``: one camera in
    viewmats / Ks) with the given colour / alpha cotangents."""

    def __init__(self, checker, sc, v_render_colors, v_render_alphas, threads=None):
        self.ck = checker
        self.sc = sc
        self.vrc = np.ascontiguousarray(v_render_colors[:1], np.float32)
        self.vra = np.ascontiguousarray(v_render_alphas[:1], np.float32)
        self.T = threads or host_threads()
        self.pool = ThreadPoolExecutor(self.T)
        self.gchunks = _chunks(sc.n, self.T)
        tiles = sc.tile_width * sc.tile_height
        owner = np.arange(tiles) % self.T
        self.masks = [(owner == k).reshape(1, sc.tile_height, sc.tile_width)
                      for k in range(min(self.T, tiles))]
        # pixel owner per thread, for assembling the forward outputs
        ty = np.arange(sc.height) // sc.tile_size
        tx = np.arange(sc.width) // sc.tile_size
        pix_owner = owner[(ty[:, None] * sc.tile_width + tx[None, :])].reshape(-1)
        self.pix_of = [np.flatnonzero(pix_owner == k) for k in range(len(self.masks))]

    def close(self):
        self.pool.shutdown()

    def _map(self, fn, items):
        return list(self.pool.map(fn, items))

    def run(self):
        """Runs the step; returns (seconds, intersections, seconds of the
        intersect pipeline (count, scan, encode, sort))."""
        ck, sc = self.ck, self.sc
        W, H, ts, tw, th = sc.width, sc.height, sc.tile_size, sc.tile_width, sc.tile_height
        N = sc.n
        view, Ks = sc.viewmats[None], sc.Ks[None]
        t0 = time.perf_counter()
        # projection forward per Gaussian chunk
        parts = self._map(lambda c: ck.proj_fwd(sc.means[None, c[0]:c[1]], view, Ks, W, H,
                                                quats=sc.quats[None, c[0]:c[1]],
                                                scales=sc.scales[None, c[0]:c[1]]),
                          self.gchunks)
        p = {k: np.concatenate([q[k] for q in parts], axis=2) for k in
             ("means2d", "depths", "conics", "radii")}
        p["compensations"] = np.zeros((0,), np.float32)
        metal_cull(p, W, H)
        # SH colour glue (dirs from the camera centre, clip(SH + 0.5, 0, 1))
        R, t = sc.viewmats[0, :3, :3], sc.viewmats[0, :3, 3]
        campos = -(R.T @ t)
        dirs = (sc.means - campos).astype(np.float32)
        dirs /= np.maximum(np.linalg.norm(dirs, axis=-1, keepdims=True), 1e-8)
        sh = self._map(lambda c: ck.sh_fwd(sc.sh_degree, dirs[c[0]:c[1]], sc.coeffs[c[0]:c[1]]),
                       self.gchunks)
        colors = np.clip(np.concatenate(sh) + 0.5, 0, 1)[None].astype(np.float32)
        # intersect: count / scan / encode / stable sort per chunk, stable merge
        m2 = p["means2d"].reshape(1, N, 2)
        rad = p["radii"].reshape(1, N, 2)
        dep = p["depths"].reshape(1, N)
        ti = time.perf_counter()
        its = self._map(lambda c: ck.isect_tile(m2[:, c[0]:c[1]], rad[:, c[0]:c[1]],
                                                dep[:, c[0]:c[1]], 1, ts, tw, th), self.gchunks)
        keys = np.concatenate([q["isect_ids"] for q in its])
        fids = np.concatenate([q["flatten_ids"] + np.int32(c[0])
                               for q, c in zip(its, self.gchunks)])
        order = np.argsort(keys, kind="stable")
        keys, fids = keys[order], fids[order].astype(np.int32)
        t_isect = time.perf_counter() - ti
        offs = ck.isect_offset(keys, 1, tw, th)
        kw = dict(means2d=m2, conics=p["conics"].reshape(1, N, 3), colors=colors,
                  opacities=sc.opacities[None], tile_offsets=offs, flatten_ids=fids,
                  width=W, height=H, tile_size=ts)
        # rasterize forward: one tile set per thread
        rfs = self._map(lambda m: ck.raster_fwd(masks=m, threads=1, **kw), self.masks)
        rf = {k: np.empty_like(rfs[0][k]) for k in rfs[0]}
        for k in rf:
            flat = rf[k].reshape(H * W, -1)
            for q, pix in zip(rfs, self.pix_of):
                flat[pix] = q[k].reshape(H * W, -1)[pix]
        # rasterize backward: one tile set per thread, gradients summed
        rbs = self._map(lambda m: ck.raster_bwd(render_alphas=rf["render_alphas"],
                                                last_ids=rf["last_ids"],
                                                v_render_colors=self.vrc,
                                                v_render_alphas=self.vra, masks=m, threads=1,
                                                **kw),
                        self.masks)
        rb = {k: self._sum([q[k] for q in rbs]) for k in rbs[0]}
        # SH backward and projection backward per Gaussian chunk
        shb = self._map(lambda c: ck.sh_bwd(sc.sh_degree, dirs[c[0]:c[1]],
                                            sc.coeffs[c[0]:c[1]], rb["v_colors"][0, c[0]:c[1]]),
                        self.gchunks)
        pbs = self._map(lambda c: ck.proj_bwd(sc.means[None, c[0]:c[1]], view, Ks, W, H,
                                        p["radii"][:, :, c[0]:c[1]], p["conics"][:, :, c[0]:c[1]],
                                        rb["v_means2d"][None, :, c[0]:c[1]],
                                        np.zeros((1, 1, c[1] - c[0]), np.float32),
                                        rb["v_conics"][None, :, c[0]:c[1]],
                                        quats=sc.quats[None, c[0]:c[1]],
                                        scales=sc.scales[None, c[0]:c[1]]), self.gchunks)
        dt = time.perf_counter() - t0
        # the step's results, for checking this driver against one-thread runs
        self.last = {"isect_ids": keys, "flatten_ids": fids, "tile_offsets": offs, "colors": colors,
                     **{"rf_" + k: v for k, v in rf.items()}, **{"rb_" + k: v for k, v in rb.items()},
                     "v_coeffs": np.concatenate([q["v_coeffs"] for q in shb]),
                     "v_means": np.concatenate([q["v_means"] for q in pbs], axis=1)}
        return dt, int(keys.size), t_isect

    def _sum(self, arrays):
        """Sum of equally shaped arrays, split across the threads."""
        out = np.empty_like(arrays[0])
        flat = [a.reshape(-1) for a in arrays]
        o = out.reshape(-1)

        def part(c):
            a, b = c
            acc = flat[0][a:b].copy()
            for f in flat[1:]:
                acc += f[a:b]
            o[a:b] = acc

        self._map(part, _chunks(o.size, self.T))
        return out
