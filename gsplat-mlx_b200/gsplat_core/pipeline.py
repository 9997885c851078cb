"""Fused training step over the gsplat_core operators.

One ``TrainingStep.run()`` is the forward and backward pass that the
reference trainers build per batch of cameras (render_sh_model and the
autograd of sh_loss_fn, scripts/test/scanner_points_training_utils.py:
1050-1122 and 2076-2119):

  projection fwd -> SH colour glue fwd -> count -> scan -> (host read of the
  intersection count) -> depth-ordered encode + tile/image radix passes
  (= encode -> stable key sort) -> tile offsets -> rasterize fwd ->
  rasterize bwd -> projection bwd -> SH glue bwd

with the cotangents of the rendered colours / alphas given.  Every stage is
a native kernel of libgsplat_b200.so called through its C ABI on one CUDA
stream; device buffers come from torch and are allocated once per shape.
The per-Gaussian gradients land in one flat buffer
``[v_means | v_quats | v_scales | v_opacities | v_coeffs]`` so that a
multi-GPU step can all-reduce them in a single collective.
"""
from __future__ import annotations

import ctypes as ct

import torch

from . import _lib
from ._lib import (IsectParams, ProjectionParams, RasterParams, SHGlueParams, check)


def _p(t):
    return None if t is None else ct.c_void_p(t.data_ptr())


def _s():
    return ct.c_void_p(torch.cuda.current_stream().cuda_stream)


# ------------------------------------------------------------- SH colour glue

def sh_colors(degree, means, viewmats, coeffs, masks=None, radii=None):
    """colors [C,N,3] = clip(SH(normalize(means - campos_c)) + 0.5, 0, 1)
    (sh_colors_for_camera, scanner_points_training_utils.py:1011-1034),
    fused into one kernel.  Entries masked out / culled get 0."""
    C = viewmats.numel() // 16
    N = means.shape[0]
    K = coeffs.shape[-2]
    out = torch.empty((C, N, 3), dtype=torch.float32, device=means.device)
    p = SHGlueParams(C, N, K, int(degree), int(masks is not None))
    check(_lib.load().gs_sh_glue_fwd(ct.byref(p), _p(means), _p(viewmats), _p(coeffs), _p(masks),
                                     _p(radii), _p(out), _s()), "sh_colors")
    return out


def sh_colors_backward(degree, means, viewmats, coeffs, masks, v_colors, v_means_accum,
                       radii=None, v_coeffs=None, skip_zero_cotangents=False, camera_groups=1):
    """Reverse mode of sh_colors as MLX autograd forms it; adds into
    v_means_accum [N,3] and returns v_coeffs [N,K,3] (summed over cameras).
    With skip_zero_cotangents, entries whose colour cotangent is zero are
    skipped (they contribute nothing) -- the visibility test for cameras
    whose radii are not at hand."""
    C = viewmats.numel() // 16
    N = means.shape[0]
    K = coeffs.shape[-2]
    if v_coeffs is None:
        v_coeffs = torch.empty_like(coeffs)
    p = SHGlueParams(C, N, K, int(degree), int(masks is not None), int(skip_zero_cotangents),
                     int(camera_groups))
    check(_lib.load().gs_sh_glue_bwd(ct.byref(p), _p(means), _p(viewmats), _p(coeffs), _p(masks),
                                     _p(radii), _p(v_colors), _p(v_means_accum), _p(v_coeffs),
                                     _s()), "sh_colors_backward")
    return v_coeffs


# ------------------------------------------------------------- training step

class TrainingStep:
    """Preallocated forward+backward of the 3DGS hot path for one batch of
    C cameras of one scene (B = 1, I = C images)."""

    def __init__(self, n, sh_degree, K, cameras, width, height, tile_size=16, eps2d=0.3,
                 near_plane=0.01, far_plane=1e10, device=None, use_background=True,
                 max_isects_per_pass=1 << 30, tile_cull=False):
        self.dev = device or torch.device("cuda", torch.cuda.current_device())
        self.N, self.deg, self.K, self.C = int(n), int(sh_degree), int(K), int(cameras)
        self.W, self.H, self.ts = int(width), int(height), int(tile_size)
        self.tw = (self.W + self.ts - 1) // self.ts
        self.th = (self.H + self.ts - 1) // self.ts
        self.eps2d, self.near, self.far = float(eps2d), float(near_plane), float(far_plane)
        self.lib = _lib.load()
        self.max_isects_per_pass = int(max_isects_per_pass)
        self.bands = 1
        f32, i32 = torch.float32, torch.int32
        C, N = self.C, self.N
        e = lambda shape, dt=f32: torch.empty(shape, dtype=dt, device=self.dev)  # noqa: E731
        # forward state
        self.means2d, self.depths = e((C, N, 2)), e((C, N))
        self.conics, self.radii = e((C, N, 3)), e((C, N, 2), i32)
        self.colors = e((C, N, 3))
        self.sbounds = e((N, 2))  # exact alpha decisions per opacity (sigma bounds)
        # the sigma bounds run on a side stream, beside the intersection
        # encode (a chain of small, latency-bound kernels)
        self.side = torch.cuda.Stream(device=self.dev)
        self.tiles_per_gauss = e((C, N), i32)
        # [intersections, bin entries of the binned encode]
        self.total = torch.zeros((2,), dtype=torch.int64, device=self.dev)
        self.total_host = torch.zeros((2,), dtype=torch.int64, pin_memory=True)
        self.tile_offsets = e((C, self.th, self.tw), i32)
        # the rasterizers' tile schedule (costliest tiles first), and the
        # forward's per-tile cost record that orders the backward
        self.tile_order = e((C * self.th * self.tw,), i32)
        self.tile_cost = e((C * self.th * self.tw,), i32)
        self.render_colors = e((C, self.H, self.W, 3))
        self.render_alphas = e((C, self.H, self.W, 1))
        self.last_ids = e((C, self.H, self.W), i32)
        self.backgrounds = torch.zeros((C, 3), dtype=f32, device=self.dev) if use_background else None
        self.v_backgrounds = e((C, 3)) if use_background else None
        # intersections (grown on demand); the binned encode needs 16-bit
        # tile coordinates, else the depth-first sorted encode runs
        self.binned = max(self.tw, self.th) <= 65535
        # opacity-aware tile culling in the binned encode (opt-in): (tile,
        # Gaussian) pairs below alpha 1/255 at every pixel centre of the tile
        # are not listed (the rasterizer would skip them at each pixel; the
        # renders are the same bit for bit, the lists shorter).  The 16x16
        # rasterizers drop such pairs themselves when they stage a batch, so
        # the step gains little from it.  Kept totals per band.
        self.tile_cull = bool(tile_cull) and self.binned
        self.kept = torch.zeros((64,), dtype=torch.int64, device=self.dev)
        self.capacity = 0
        self.sort_ws = torch.empty((0,), dtype=torch.uint8, device=self.dev)
        self.m = 0
        self.bins = 0
        # backward state
        self.v_means2d, self.v_conics = e((C, N, 2)), e((C, N, 3))
        self.v_colors = e((C, N, 3))
        self.v_depths = torch.zeros((C, N), dtype=f32, device=self.dev)
        sizes = [3 * N, 4 * N, 3 * N, N, self.K * 3 * N]
        self.grad_flat = e((sum(sizes),))
        views = torch.split(self.grad_flat, sizes)
        self.v_means = views[0].view(N, 3)
        self.v_quats = views[1].view(N, 4)
        self.v_scales = views[2].view(N, 3)
        self.v_opacities = views[3].view(N)
        self.v_coeffs = views[4].view(N, self.K, 3)
        n_tiles = self.tw * self.th
        self.key_bits = 32 + self.lib.gs_floor_log2_plus_one(n_tiles) + \
            self.lib.gs_floor_log2_plus_one(C)
        self.events = None

    def _ensure_capacity(self, m, bins=0):
        """Grows the intersection buffers and the workspace of the encode;
        True when the workspace was reallocated."""
        e = lambda shape, dt: torch.empty(shape, dtype=dt, device=self.dev)  # noqa: E731
        grew = False
        if m > self.capacity:
            cap = max(int(m * 1.25) + 1024, 1 << 16)
            self.sorted_ids = e((cap,), torch.int64)
            self.sorted_flatten = e((cap,), torch.int32)
            self.capacity = cap
            if not self.binned:
                self.sort_ws = e((self.lib.gs_isect_tile_encode_sorted_workspace_size(
                    self.C * self.N, cap),), torch.uint8)
                grew = True
        if self.binned:
            # sized for every tile row: a band needs less
            ip = IsectParams(self.C, self.N, self.ts, self.tw, self.th, 0, 0)
            need = self.lib.gs_isect_tile_encode_binned_workspace_size(ct.byref(ip), bins)
            if need > self.sort_ws.numel():
                self.sort_ws = e((int(need * 1.25) + (1 << 20),), torch.uint8)
                grew = True
        return grew

    def _mark(self, name):
        if self.events is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self.events.append((name, ev))

    def _side_mark(self):
        """A timing event on the side stream (None when not timing)."""
        if self.events is None:
            return None
        ev = torch.cuda.Event(enable_timing=True)
        ev.record(self.side)
        return ev

    def _side_span(self, name, ev0):
        """Records the side-stream stage that began at ``ev0``."""
        ev1 = self._side_mark()
        if ev0 is not None and ev1 is not None:
            self.side_spans.append((name, ev0, ev1))

    def run(self, means, quats, scales, opacities, coeffs, viewmats, Ks, v_render_colors,
            v_render_alphas, sh_backward=True, colors=None, target=None, after_raster=None):
        """Forward and backward; returns the flat gradient buffer (a view of
        self.grad_flat) and the intersection count of this step.

        With ``sh_backward=False`` the SH colour glue backward is left to the
        caller: v_coeffs is not written and v_means holds the projection part
        only, while ``self.v_colors`` holds the colour cotangents (the camera-
        sharded step exchanges those instead of the SH gradients).

        ``colors`` [C,N,3] (or [N,3] for one camera) replaces the SH colour
        glue: the rasterizer uses them directly, no SH glue runs and
        ``self.v_colors`` holds their gradient (the image-fitting trainer).
        ``target`` [C,H,W,3] replaces the given cotangents by those of the
        L2 loss mean((render - target)^2), whose value lands in the device
        scalar ``self.loss``.

        ``after_raster()`` is called once the rasterizer backward of every
        band is queued (``self.v_colors`` complete on the stream), before the
        projection backward: the camera-sharded step starts its colour
        exchange there.

        When the step has more than ``max_isects_per_pass`` intersections
        (the int32 offsets of the operator surface cap one pass at 2^31), the
        image is processed in bands of tile rows: each band gets its own
        count / sorted encode (with its tile offsets) / rasterize forward and
        backward (accumulating into the same gradients), all bit-identical to
        one pass over the rows of the band; projection and SH run once."""
        L, s = self.lib, _s()
        C, N = self.C, self.N
        self._mark("start")
        pp = ProjectionParams(1, C, N, self.W, self.H, self.eps2d, self.near, self.far, 0.0, 0, 0,
                              0, 0)
        check(L.gs_projection_fwd(ct.byref(pp), _p(means), None, _p(quats), _p(scales), None,
                                  _p(viewmats), _p(Ks), _p(self.means2d), _p(self.depths),
                                  _p(self.conics), None, _p(self.radii), s), "projection_fwd")
        self._mark("projection_fwd")
        projected = torch.cuda.Event()
        projected.record()
        self.side_spans = []
        bounded = None
        gp = SHGlueParams(C, N, self.K, self.deg, 0)
        glue_pending = colors is None
        if glue_pending:
            colors = self.colors
        else:
            sh_backward = False
        # the rasterizer and the culled encode read the [N] opacities of
        # every camera in place and sum their gradient over the cameras
        opac, v_opac = opacities, self.v_opacities
        m_total = 0
        bands = [(0, 0)]  # (0, 0): every tile row in one pass
        b = 0
        while b < len(bands):
            y0, y1 = bands[b]
            ip = IsectParams(C, N, self.ts, self.tw, self.th, y0, y1)
            # the projection culls depths below its near plane: with a
            # positive near plane every visible depth is positive
            ip.positive_depths = int(self.near > 0.0)
            ip.shared_opacities = 1
            check(L.gs_isect_tile_count_totals(ct.byref(ip), _p(self.means2d), _p(self.radii),
                                               _p(self.tiles_per_gauss), _p(self.total), s),
                  "isect_count")
            # the host read of the totals: kernel stores into the pinned
            # buffer, not a copy that could queue behind a download
            check(L.gs_store_to_host_i64(_p(self.total), _p(self.total_host), 2, s),
                  "isect_count")
            self._mark("isect_count")
            counted = torch.cuda.Event()
            counted.record()
            if glue_pending:
                # The SH colours are first needed by the rasterizer: the
                # device computes them while the host reads the totals.  (On
                # the side stream, beside the encode, they slowed the encode
                # by about their own time: no gain.)
                check(L.gs_sh_glue_fwd(ct.byref(gp), _p(means), _p(viewmats), _p(coeffs), None,
                                       _p(self.radii), _p(self.colors), s), "sh_glue_fwd")
                self._mark("sh_fwd")
                glue_pending = False
            counted.synchronize()  # the reference's host read of the total
            if bounded is None:
                # launched now, the bounds kernel runs beside the encode
                self.side.wait_event(projected)
                t0 = self._side_mark()
                check(L.gs_rasterize_sigma_bounds(N, _p(opacities), _p(self.radii), C,
                                                  _p(self.sbounds),
                                                  ct.c_void_p(self.side.cuda_stream)),
                      "rasterize_sigma_bounds")
                self._side_span("sigma_bounds", t0)
                bounded = torch.cuda.Event()
                bounded.record(self.side)
            m, bins = (int(v) for v in self.total_host.tolist())
            if m > self.max_isects_per_pass and y1 == 0:
                # too many intersections for one pass (int32 offsets, memory):
                # bands of tile rows, each with its own intersection pass
                if target is not None:
                    raise RuntimeError("the L2-target mode renders in one pass; "
                                       f"{m} intersections exceed max_isects_per_pass")
                rows = max(1, int(self.th * self.max_isects_per_pass // (2 * m)))
                bands = [(r, min(r + rows, self.th)) for r in range(0, self.th, rows)]
                continue
            if m >= 2 ** 31:
                raise RuntimeError(f"{m} intersections exceed the int32 index range"
                                   + (f" in tile rows {y0}..{y1}" if y1 else ""))
            grew = self._ensure_capacity(m, bins)
            self.m, self.bins = m, bins
            m_total += m
            if self.binned and self.tile_cull:
                # sorted, tile-culled intersections (the last places of the
                # lists) and the band's tile offsets in one call
                if b >= self.kept.numel():
                    self.kept = torch.zeros((2 * len(bands),), dtype=torch.int64, device=self.dev)
                check(L.gs_isect_tile_encode_binned_culled(
                    ct.byref(ip), _p(self.means2d), _p(self.radii), _p(self.depths),
                    _p(self.conics), _p(opac), m, bins, _p(self.sorted_ids),
                    _p(self.sorted_flatten), _p(self.tile_offsets),
                    ct.c_void_p(self.kept.data_ptr() + 8 * b), _p(self.sort_ws),
                    self.sort_ws.numel(), s), "isect_encode_sort")
                self._mark("isect_encode_sort")
            elif self.binned:
                # sorted intersections and the band's tile offsets in one call
                check(L.gs_isect_tile_encode_binned(ct.byref(ip), _p(self.means2d),
                                                    _p(self.radii), _p(self.depths), m, bins,
                                                    _p(self.sorted_ids), _p(self.sorted_flatten),
                                                    _p(self.tile_offsets), _p(self.sort_ws),
                                                    self.sort_ws.numel(), s),
                      "isect_encode_sort")
                self._mark("isect_encode_sort")
            else:
                # bands after the first reuse the depth order of the elements
                # left in the workspace (unless it was just reallocated)
                ip.reuse_depth_order = int(not grew and b > 0 and y1 > 0)
                check(L.gs_isect_tile_encode_sorted(ct.byref(ip), _p(self.means2d),
                                                    _p(self.radii), _p(self.depths),
                                                    _p(self.tiles_per_gauss), m,
                                                    _p(self.sorted_ids), _p(self.sorted_flatten),
                                                    _p(self.sort_ws), self.sort_ws.numel(), s),
                      "isect_encode_sort")
                self._mark("isect_encode_sort")
                r0, r1 = (y0, y1) if y1 else (0, self.th)
                check(L.gs_isect_offset_rows(m, _p(self.sorted_ids), C, self.tw, self.th, r0, r1,
                                             _p(self.tile_offsets), s), "isect_offset")
                self._mark("isect_offset")
            rp = RasterParams(C, N, 3, self.W, self.H, self.ts, self.tw, self.th, m,
                              int(self.backgrounds is not None), 0, 0, y0, y1, int(b > 0), 1,
                              _p(self.sbounds), _p(self.tile_order), _p(self.tile_cost))
            torch.cuda.current_stream().wait_event(bounded)
            check(L.gs_rasterize_fwd(ct.byref(rp), _p(self.means2d), _p(self.conics),
                                     _p(colors), _p(opac), _p(self.backgrounds), None,
                                     _p(self.tile_offsets), _p(self.sorted_flatten),
                                     _p(self.render_colors), _p(self.render_alphas),
                                     _p(self.last_ids), s), "rasterize_fwd")
            self._mark("rasterize_fwd")
            if target is not None:
                if not hasattr(self, "loss"):
                    self.loss = torch.zeros((1,), dtype=torch.float32, device=self.dev)
                    self.v_rc_loss = torch.empty_like(self.render_colors)
                    self.v_ra_zero = torch.zeros_like(self.render_alphas)
                check(L.gs_l2_loss_grad(self.render_colors.numel(), _p(self.render_colors),
                                        _p(target), _p(self.v_rc_loss), _p(self.loss), s),
                      "l2_loss")
                v_render_colors, v_render_alphas = self.v_rc_loss, self.v_ra_zero
                self._mark("loss")
            check(L.gs_rasterize_bwd(ct.byref(rp), _p(self.means2d), _p(self.conics),
                                     _p(colors), _p(opac), _p(self.backgrounds), None,
                                     _p(self.tile_offsets), _p(self.sorted_flatten),
                                     _p(self.render_alphas), _p(self.last_ids),
                                     _p(v_render_colors), _p(v_render_alphas), None,
                                     _p(self.v_means2d), _p(self.v_conics), _p(self.v_colors),
                                     _p(v_opac), _p(self.v_backgrounds), s), "rasterize_bwd")
            self._mark("rasterize_bwd")
            b += 1
        m = m_total
        self.m_total = m_total
        self.bands = len(bands)
        if after_raster is not None:
            after_raster()
        check(L.gs_projection_bwd(ct.byref(pp), _p(means), None, _p(quats), _p(scales),
                                  _p(viewmats), _p(Ks), _p(self.radii), _p(self.conics), None,
                                  _p(self.v_means2d), _p(self.v_depths), _p(self.v_conics), None,
                                  _p(self.v_means), None, _p(self.v_quats), _p(self.v_scales),
                                  None, s), "projection_bwd")
        self._mark("projection_bwd")
        if not sh_backward:
            return self.grad_flat, m
        check(L.gs_sh_glue_bwd(ct.byref(gp), _p(means), _p(viewmats), _p(coeffs), None,
                               _p(self.radii), _p(self.v_colors), _p(self.v_means),
                               _p(self.v_coeffs), s), "sh_glue_bwd")
        self._mark("sh_bwd")
        return self.grad_flat, m

    def check(self):
        """Waits for the step and raises if a bounded on-device wait of the
        intersection sort gave up (its output would be invalid)."""
        if self.m > 0 and self.binned:
            check(self.lib.gs_isect_tile_encode_binned_check(self.bins, _p(self.sort_ws), _s()),
                  "isect_encode_sort")
        elif self.m > 0:
            check(self.lib.gs_isect_tile_encode_sorted_check(
                self.C * self.N, self.m, _p(self.sort_ws), _s()), "isect_encode_sort")

    def kept_isects(self) -> int:
        """Intersections the last step's rasterizer passes walked: the
        tile-culled totals of its bands (a host read), else the counted
        total."""
        if not self.tile_cull:
            return self.m_total
        return int(self.kept[:self.bands].sum().item())

    def gradients(self):
        return {"v_means": self.v_means, "v_quats": self.v_quats, "v_scales": self.v_scales,
                "v_opacities": self.v_opacities, "v_coeffs": self.v_coeffs}
