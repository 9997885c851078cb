"""numpy front-end over the two CPU checkers (TEST INFRASTRUCTURE ONLY).

* ``Oracle``    -> ``oracle/liboracle.so``: the C restatement in
  ``gsplat_oracle.c`` (always available once ``make -C oracle`` ran).
* ``Reference`` -> ``oracle/_ref/libgsplat_ref.so``: the reference's own
  ``gsplat_core/*.cpp`` eval_cpu code compiled against ``mlx_shim`` (only
  where it was built; ``Reference.available()`` says so).

Both expose the same methods with the same argument meaning, mirroring the
reference op front-ends (gsplat_core/include/gsplat_*.h) and the binding's
dict keys (gsplat_core/binding/binding.cpp).  Only tests/, smoke() and the
CPU-baseline leg of bench.py use this module; the product never does.
"""
from __future__ import annotations

import ctypes as ct
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(_HERE, "liboracle.so")
REF_SO = os.path.join(_HERE, "_ref", "libgsplat_ref.so")
REF_CUDA_SO = os.path.join(_HERE, "_ref", "libgsplat_ref_cuda.so")

_vp = ct.c_void_p
_i = ct.c_int
_i64 = ct.c_int64
_f = ct.c_float


def _p(a):
    return None if a is None else a.ctypes.data_as(_vp)


def _f32(a):
    return None if a is None else np.ascontiguousarray(a, dtype=np.float32)


def _i32(a):
    return None if a is None else np.ascontiguousarray(a, dtype=np.int32)


def _u8(a):
    return None if a is None else np.ascontiguousarray(a, dtype=np.uint8)


def raster_threads(bytes_per_thread: int = 0) -> int:
    """Worker threads of the oracle's rasterizer: every core this process
    may use (GSPLAT_ORACLE_THREADS overrides), fewer when each backward
    worker's private gradient copy would take more than 4 GB in total."""
    n = int(os.environ.get("GSPLAT_ORACLE_THREADS", "0")) or len(os.sched_getaffinity(0))
    if bytes_per_thread > 0:
        n = min(n, max(1, int(4e9 // bytes_per_thread)))
    return max(1, min(n, 256))


def _check(rc, lib, what):
    if rc != 0:
        msg = ""
        if hasattr(lib, "ref_last_error"):
            msg = lib.ref_last_error().decode()
        raise RuntimeError(f"{what} failed ({rc}) {msg}")


class _Common:
    """Shape handling shared by both checkers."""

    lib = None

    # ---------------- quat/scale -> covariance ----------------
    def qs2c_fwd(self, quats, scales, compute_covar=True, compute_preci=True,
                 triu=True):
        quats, scales = _f32(quats), _f32(scales)
        n = quats.size // 4
        prefix = quats.shape[:-1]
        tail = (6,) if triu else (3, 3)
        cov = np.zeros(prefix + tail, np.float32) if compute_covar else np.zeros((0,), np.float32)
        pre = np.zeros(prefix + tail, np.float32) if compute_preci else np.zeros((0,), np.float32)
        self._qs2c_fwd(n, quats, scales, compute_covar, compute_preci, triu,
                       cov if compute_covar else None, pre if compute_preci else None)
        return {"covars": cov, "precis": pre}

    def qs2c_bwd(self, quats, scales, v_covars=None, v_precis=None, triu=True):
        quats, scales = _f32(quats), _f32(scales)
        n = quats.size // 4
        vq = np.zeros(quats.shape, np.float32)
        vs = np.zeros(scales.shape, np.float32)
        self._qs2c_bwd(n, quats, scales, _f32(v_covars), _f32(v_precis), triu, vq, vs)
        return {"v_quats": vq, "v_scales": vs}

    # ---------------- projection ----------------
    def proj_fwd(self, means, viewmats, Ks, width, height, covars=None,
                 quats=None, scales=None, opacities=None, eps2d=0.3,
                 near_plane=0.01, far_plane=1e10, radius_clip=0.0,
                 calc_compensations=False, camera_model=0):
        means = _f32(means)
        viewmats = _f32(viewmats)
        B = int(np.prod(means.shape[:-2])) if means.ndim > 2 else 1
        N = means.shape[-2]
        C = viewmats.shape[-3]
        prefix = means.shape[:-2] + (C, N)
        out = {
            "means2d": np.zeros(prefix + (2,), np.float32),
            "depths": np.zeros(prefix, np.float32),
            "conics": np.zeros(prefix + (3,), np.float32),
            "compensations": np.zeros(prefix if calc_compensations else (0,), np.float32),
            "radii": np.zeros(prefix + (2,), np.int32),
        }
        self._proj_fwd(B, C, N, means, _f32(covars), _f32(quats), _f32(scales),
                       _f32(opacities), viewmats, _f32(Ks), width, height, eps2d,
                       near_plane, far_plane, radius_clip, calc_compensations,
                       camera_model, out["means2d"], out["depths"], out["conics"],
                       out["compensations"] if calc_compensations else None,
                       out["radii"])
        return out

    def proj_bwd(self, means, viewmats, Ks, width, height, radii, conics,
                 v_means2d, v_depths, v_conics, covars=None, quats=None,
                 scales=None, compensations=None, v_compensations=None,
                 eps2d=0.3, viewmats_requires_grad=False):
        means = _f32(means)
        viewmats = _f32(viewmats)
        B = int(np.prod(means.shape[:-2])) if means.ndim > 2 else 1
        N = means.shape[-2]
        C = viewmats.shape[-3]
        if compensations is not None and np.asarray(compensations).size == 0:
            compensations = None
        if v_compensations is not None and np.asarray(v_compensations).size == 0:
            v_compensations = None
        out = {"v_means": np.zeros(means.shape, np.float32)}
        if covars is not None:
            out["v_covars"] = np.zeros(np.shape(covars), np.float32)
        else:
            out["v_quats"] = np.zeros(np.shape(quats), np.float32)
            out["v_scales"] = np.zeros(np.shape(scales), np.float32)
        if viewmats_requires_grad:
            out["v_viewmats"] = np.zeros(viewmats.shape, np.float32)
        self._proj_bwd(B, C, N, means, _f32(covars), _f32(quats), _f32(scales),
                       viewmats, _f32(Ks), width, height, eps2d, _i32(radii),
                       _f32(conics), _f32(compensations), _f32(v_means2d),
                       _f32(v_depths), _f32(v_conics), _f32(v_compensations),
                       out["v_means"], out.get("v_covars"), out.get("v_quats"),
                       out.get("v_scales"), out.get("v_viewmats"))
        return out

    # ---------------- spherical harmonics ----------------
    def sh_fwd(self, degree, dirs, coeffs, masks=None):
        dirs, coeffs = _f32(dirs), _f32(coeffs)
        n = dirs.size // 3
        K = coeffs.shape[-2]
        colors = np.zeros(dirs.shape, np.float32)
        self._sh_fwd(n, K, degree, dirs, coeffs, _u8(masks), colors)
        return colors

    def sh_bwd(self, degree, dirs, coeffs, v_colors, masks=None,
               compute_v_dirs=True):
        dirs, coeffs = _f32(dirs), _f32(coeffs)
        n = dirs.size // 3
        K = coeffs.shape[-2]
        v_dirs = np.zeros(dirs.shape, np.float32) if compute_v_dirs else None
        v_coeffs = np.zeros(coeffs.shape, np.float32)
        self._sh_bwd(n, K, degree, dirs, coeffs, _u8(masks), _f32(v_colors),
                     compute_v_dirs, v_dirs, v_coeffs)
        out = {"v_coeffs": v_coeffs}
        if compute_v_dirs:
            out["v_dirs"] = v_dirs
        return out

    # ---------------- intersection ----------------
    def isect_offset(self, isect_ids, I, tile_width, tile_height):
        ids = np.ascontiguousarray(isect_ids, dtype=np.int64)
        out = np.zeros((I, tile_height, tile_width), np.int32)
        self._isect_offset(ids.size, ids, I, tile_width, tile_height, out)
        return out

    # ---------------- rasterize ----------------
    @staticmethod
    def _raster_dims(means2d, colors, tile_offsets):
        tile_offsets = np.asarray(tile_offsets)
        th, tw = tile_offsets.shape[-2], tile_offsets.shape[-1]
        I = tile_offsets.size // (th * tw)
        N = np.asarray(means2d).shape[-2]
        ch = np.asarray(colors).shape[-1]
        return I, N, ch, th, tw

    def raster_fwd(self, means2d, conics, colors, opacities, tile_offsets,
                   flatten_ids, width, height, tile_size, backgrounds=None,
                   masks=None, threads=None):
        """threads: worker threads of the C restatement (default: every
        core); the results do not depend on it."""
        I, N, ch, th, tw = self._raster_dims(means2d, colors, tile_offsets)
        prefix = np.asarray(tile_offsets).shape[:-2]
        flatten_ids = _i32(flatten_ids)
        out = {
            "render_colors": np.zeros(prefix + (height, width, ch), np.float32),
            "render_alphas": np.zeros(prefix + (height, width, 1), np.float32),
            "last_ids": np.zeros(prefix + (height, width), np.int32),
        }
        self._raster_fwd(I, N, ch, _f32(means2d), _f32(conics), _f32(colors),
                         _f32(opacities), _f32(backgrounds), _u8(masks), width,
                         height, tile_size, tw, th, _i32(tile_offsets),
                         flatten_ids.size, flatten_ids, out["render_colors"],
                         out["render_alphas"], out["last_ids"], threads)
        return out

    def raster_bwd(self, means2d, conics, colors, opacities, tile_offsets,
                   flatten_ids, width, height, tile_size, render_alphas,
                   last_ids, v_render_colors, v_render_alphas,
                   backgrounds=None, masks=None, absgrad=False, threads=None):
        """threads: worker threads of the C restatement (default: every
        core, fewer for very large gradient buffers).  Each worker sums its
        tiles' contributions separately, so the gradients depend on the
        thread count through the order of the float additions only;
        threads=1 gives the reference's tile order."""
        I, N, ch, th, tw = self._raster_dims(means2d, colors, tile_offsets)
        flatten_ids = _i32(flatten_ids)
        shape2 = np.asarray(means2d).shape
        out = {
            "v_means2d": np.zeros(shape2, np.float32),
            "v_conics": np.zeros(np.asarray(conics).shape, np.float32),
            "v_colors": np.zeros(np.asarray(colors).shape, np.float32),
            "v_opacities": np.zeros(np.asarray(opacities).shape, np.float32),
        }
        if absgrad:
            out["v_means2d_abs"] = np.zeros(shape2, np.float32)
        if backgrounds is not None:
            out["v_backgrounds"] = np.zeros(np.asarray(backgrounds).shape, np.float32)
        self._raster_bwd(I, N, ch, _f32(means2d), _f32(conics), _f32(colors),
                         _f32(opacities), _f32(backgrounds), _u8(masks), width, height,
                         tile_size, tw, th, _i32(tile_offsets), flatten_ids.size,
                         flatten_ids, _f32(render_alphas), _i32(last_ids),
                         _f32(v_render_colors), _f32(v_render_alphas),
                         absgrad, out.get("v_means2d_abs"), out["v_means2d"],
                         out["v_conics"], out["v_colors"], out["v_opacities"],
                         out.get("v_backgrounds"), threads)
        return out


class Oracle(_Common):
    """The C restatement (``gsplat_oracle.c``)."""

    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            raise RuntimeError(f"oracle library missing: {path} (run make -C oracle)")
        L = ct.CDLL(path)
        self.lib = L
        L.orc_qs2c_fwd.argtypes = [_i64, _vp, _vp, _i, _i, _i, _vp, _vp]
        L.orc_qs2c_bwd.argtypes = [_i64, _vp, _vp, _vp, _vp, _i, _vp, _vp]
        L.orc_proj_fwd.argtypes = [_i, _i, _i] + [_vp] * 7 + [_i, _i, _f, _f, _f, _f, _i, _i] + [_vp] * 5
        L.orc_proj_bwd.argtypes = [_i, _i, _i] + [_vp] * 6 + [_i, _i, _f] + [_vp] * 12
        L.orc_sh_fwd.argtypes = [_i64, _i, _i, _vp, _vp, _vp, _vp]
        L.orc_sh_bwd.argtypes = [_i64, _i, _i, _vp, _vp, _vp, _vp, _vp, _vp]
        L.orc_isect_count.argtypes = [_i, _i, _vp, _vp, _i, _i, _i, _vp]
        L.orc_isect_scan.argtypes = [_i64, _vp, _vp]
        L.orc_isect_scan.restype = _i64
        L.orc_isect_encode.argtypes = [_i, _i, _vp, _vp, _vp, _vp, _i, _i, _i, _i64, _vp, _vp]
        L.orc_isect_sort.argtypes = [_i64, _vp, _vp, _vp, _vp]
        L.orc_isect_offset.argtypes = [_i64, _vp, _i, _i, _i, _vp]
        L.orc_raster_fwd.argtypes = [_i, _i, _i] + [_vp] * 6 + [_i] * 5 + [_vp, _i64] + [_vp] * 4 + [_i]
        L.orc_raster_bwd.argtypes = [_i, _i, _i] + [_vp] * 6 + [_i] * 5 + [_vp, _i64] + [_vp] * 11 + [_i]
        L.orc_sh_glue_fwd.argtypes = [_i, _i, _i, _i, _vp, _vp, _vp, _vp, _vp]
        L.orc_sh_glue_bwd.argtypes = [_i, _i, _i, _i, _vp, _vp, _vp, _vp, _vp, _vp, _vp]

    def _qs2c_fwd(self, n, q, s, cc, cp, triu, cov, pre):
        _check(self.lib.orc_qs2c_fwd(n, _p(q), _p(s), int(cc), int(cp), int(triu), _p(cov), _p(pre)), self.lib, "qs2c_fwd")

    def _qs2c_bwd(self, n, q, s, vc, vp, triu, vq, vs):
        _check(self.lib.orc_qs2c_bwd(n, _p(q), _p(s), _p(vc), _p(vp), int(triu), _p(vq), _p(vs)), self.lib, "qs2c_bwd")

    def _proj_fwd(self, B, C, N, means, covars, quats, scales, opac, view, Ks,
                  W, H, eps2d, near, far, rclip, comp, cam, m2, d, con, cmp, radii):
        _check(self.lib.orc_proj_fwd(B, C, N, _p(means), _p(covars), _p(quats), _p(scales), _p(opac),
                                     _p(view), _p(Ks), W, H, eps2d, near, far, rclip, int(comp), cam,
                                     _p(m2), _p(d), _p(con), _p(cmp), _p(radii)), self.lib, "proj_fwd")

    def _proj_bwd(self, B, C, N, means, covars, quats, scales, view, Ks, W, H, eps2d,
                  radii, conics, comps, vm2, vd, vcon, vcomp, vmeans, vcov, vq, vs, vview):
        _check(self.lib.orc_proj_bwd(B, C, N, _p(means), _p(covars), _p(quats), _p(scales), _p(view),
                                     _p(Ks), W, H, eps2d, _p(radii), _p(conics), _p(comps), _p(vm2),
                                     _p(vd), _p(vcon), _p(vcomp), _p(vmeans), _p(vcov), _p(vq), _p(vs),
                                     _p(vview)), self.lib, "proj_bwd")

    def _sh_fwd(self, n, K, deg, dirs, coeffs, masks, colors):
        _check(self.lib.orc_sh_fwd(n, K, deg, _p(dirs), _p(coeffs), _p(masks), _p(colors)), self.lib, "sh_fwd")

    def _sh_bwd(self, n, K, deg, dirs, coeffs, masks, vcol, cvd, vdirs, vco):
        _check(self.lib.orc_sh_bwd(n, K, deg, _p(dirs), _p(coeffs), _p(masks), _p(vcol),
                                   _p(vdirs) if cvd else None, _p(vco)), self.lib, "sh_bwd")

    def isect_tile(self, means2d, radii, depths, I, tile_size, tile_width,
                   tile_height, sort=True):
        means2d, radii, depths = _f32(means2d), _i32(radii), _f32(depths)
        N = depths.size // I
        tpg = np.zeros(depths.shape, np.int32)
        _check(self.lib.orc_isect_count(I, N, _p(means2d), _p(radii), tile_size, tile_width,
                                        tile_height, _p(tpg)), self.lib, "isect_count")
        offs = np.zeros(depths.size, np.int32)
        m = self.lib.orc_isect_scan(tpg.size, _p(tpg), _p(offs))
        ids = np.zeros(m, np.int64)
        fids = np.zeros(m, np.int32)
        _check(self.lib.orc_isect_encode(I, N, _p(means2d), _p(radii), _p(depths), _p(offs),
                                         tile_size, tile_width, tile_height, m, _p(ids), _p(fids)),
               self.lib, "isect_encode")
        if sort:
            sids = np.zeros(m, np.int64)
            sf = np.zeros(m, np.int32)
            _check(self.lib.orc_isect_sort(m, _p(ids), _p(fids), _p(sids), _p(sf)), self.lib, "isect_sort")
            ids, fids = sids, sf
        return {"tiles_per_gauss": tpg, "isect_ids": ids, "flatten_ids": fids}

    def isect_scan(self, counts):
        counts = _i32(counts).ravel()
        offs = np.zeros(counts.size, np.int32)
        total = self.lib.orc_isect_scan(counts.size, _p(counts), _p(offs))
        return offs, int(total)

    def isect_sort(self, isect_ids, flatten_ids):
        ids = np.ascontiguousarray(isect_ids, dtype=np.int64)
        fids = _i32(flatten_ids)
        sids = np.zeros_like(ids)
        sf = np.zeros_like(fids)
        _check(self.lib.orc_isect_sort(ids.size, _p(ids), _p(fids), _p(sids), _p(sf)), self.lib, "isect_sort")
        return sids, sf

    def _isect_offset(self, m, ids, I, tw, th, out):
        _check(self.lib.orc_isect_offset(m, _p(ids), I, tw, th, _p(out)), self.lib, "isect_offset")

    def _raster_fwd(self, I, N, ch, m2, con, col, op, bg, masks, W, H, ts, tw, th,
                    toff, m, fids, rc, ra, li, threads=None):
        _check(self.lib.orc_raster_fwd(I, N, ch, _p(m2), _p(con), _p(col), _p(op), _p(bg), _p(masks),
                                       W, H, ts, tw, th, _p(toff), m, _p(fids), _p(rc), _p(ra), _p(li),
                                       threads or raster_threads()), self.lib, "raster_fwd")

    def _raster_bwd(self, I, N, ch, m2, con, col, op, bg, masks, W, H, ts, tw, th,
                    toff, m, fids, ra, li, vrc, vra, absgrad, vabs, vm2, vcon, vcol, vop, vbg,
                    threads=None):
        per_thread = 4 * I * N * (6 + ch + (2 if absgrad else 0))
        _check(self.lib.orc_raster_bwd(I, N, ch, _p(m2), _p(con), _p(col), _p(op), _p(bg), _p(masks),
                                       W, H, ts, tw, th, _p(toff), m, _p(fids), _p(ra), _p(li), _p(vrc),
                                       _p(vra), _p(vabs) if absgrad else None, _p(vm2), _p(vcon),
                                       _p(vcol), _p(vop), _p(vbg), threads or raster_threads(per_thread)),
               self.lib, "raster_bwd")

    # ---------------- SH training glue (oracle only) ----------------
    def sh_glue_fwd(self, degree, means, viewmats, coeffs, masks=None):
        means, viewmats, coeffs = _f32(means), _f32(viewmats), _f32(coeffs)
        N = means.size // 3
        C = viewmats.size // 16
        K = coeffs.shape[-2]
        colors = np.zeros((C, N, 3), np.float32)
        _check(self.lib.orc_sh_glue_fwd(C, N, K, degree, _p(means), _p(viewmats), _p(coeffs),
                                        _p(_u8(masks)), _p(colors)), self.lib, "sh_glue_fwd")
        return colors

    def sh_glue_bwd(self, degree, means, viewmats, coeffs, v_colors, masks=None):
        means, viewmats, coeffs = _f32(means), _f32(viewmats), _f32(coeffs)
        N = means.size // 3
        C = viewmats.size // 16
        K = coeffs.shape[-2]
        vm = np.zeros((N, 3), np.float32)
        vco = np.zeros((N, K, 3), np.float32)
        _check(self.lib.orc_sh_glue_bwd(C, N, K, degree, _p(means), _p(viewmats), _p(coeffs),
                                        _p(_u8(masks)), _p(_f32(v_colors)), _p(vm), _p(vco)),
               self.lib, "sh_glue_bwd")
        return {"v_means": vm, "v_coeffs": vco}


class Reference(_Common):
    """The reference's own eval_cpu code, built by ``make -C oracle ref``."""

    @staticmethod
    def available(path: str = REF_SO) -> bool:
        return os.path.exists(path)

    def __init__(self, path: str = REF_SO):
        if not os.path.exists(path):
            raise RuntimeError(f"reference build missing: {path} (run make -C oracle ref)")
        L = ct.CDLL(path)
        self.lib = L
        L.ref_last_error.restype = ct.c_char_p
        L.ref_qs2c_fwd.argtypes = [_vp, _vp, _i, _i, _i, _i, _vp, _vp]
        L.ref_qs2c_bwd.argtypes = [_vp, _vp, _vp, _vp, _i, _i, _vp, _vp]
        L.ref_proj_fwd.argtypes = [_i, _i, _i] + [_vp] * 7 + [_i, _i, _f, _f, _f, _f, _i, _i] + [_vp] * 5
        L.ref_proj_bwd.argtypes = [_i, _i, _i] + [_vp] * 6 + [_i, _i, _f] + [_vp] * 7 + [_i] + [_vp] * 5
        L.ref_sh_fwd.argtypes = [_i, _i, _i, _vp, _vp, _vp, _vp]
        L.ref_sh_bwd.argtypes = [_i, _i, _i, _vp, _vp, _vp, _vp, _i, _vp, _vp]
        L.ref_isect_tile.argtypes = [_i, _i, _vp, _vp, _vp, _i, _i, _i, _i, _i64, _vp, _vp, _vp, _vp]
        L.ref_isect_offset.argtypes = [_i64, _vp, _i, _i, _i, _vp]
        L.ref_raster_fwd.argtypes = [_i, _i, _i] + [_vp] * 6 + [_i] * 5 + [_vp, _i64] + [_vp] * 4
        L.ref_raster_bwd.argtypes = [_i, _i, _i] + [_vp] * 6 + [_i] * 5 + [_vp, _i64] + [_vp] * 5 + [_i] + [_vp] * 6

    def _qs2c_fwd(self, n, q, s, cc, cp, triu, cov, pre):
        _check(self.lib.ref_qs2c_fwd(_p(q), _p(s), n, int(cc), int(cp), int(triu), _p(cov), _p(pre)), self.lib, "ref qs2c_fwd")

    def _qs2c_bwd(self, n, q, s, vc, vp, triu, vq, vs):
        _check(self.lib.ref_qs2c_bwd(_p(q), _p(s), _p(vc), _p(vp), n, int(triu), _p(vq), _p(vs)), self.lib, "ref qs2c_bwd")

    def _proj_fwd(self, B, C, N, means, covars, quats, scales, opac, view, Ks,
                  W, H, eps2d, near, far, rclip, comp, cam, m2, d, con, cmp, radii):
        _check(self.lib.ref_proj_fwd(B, C, N, _p(means), _p(covars), _p(quats), _p(scales), _p(opac),
                                     _p(view), _p(Ks), W, H, eps2d, near, far, rclip, int(comp), cam,
                                     _p(m2), _p(d), _p(con), _p(cmp), _p(radii)), self.lib, "ref proj_fwd")

    def _proj_bwd(self, B, C, N, means, covars, quats, scales, view, Ks, W, H, eps2d,
                  radii, conics, comps, vm2, vd, vcon, vcomp, vmeans, vcov, vq, vs, vview):
        _check(self.lib.ref_proj_bwd(B, C, N, _p(means), _p(covars), _p(quats), _p(scales), _p(view),
                                     _p(Ks), W, H, eps2d, _p(radii), _p(conics), _p(comps), _p(vm2),
                                     _p(vd), _p(vcon), _p(vcomp), int(vview is not None), _p(vmeans),
                                     _p(vcov), _p(vq), _p(vs), _p(vview)), self.lib, "ref proj_bwd")

    def _sh_fwd(self, n, K, deg, dirs, coeffs, masks, colors):
        _check(self.lib.ref_sh_fwd(n, K, deg, _p(dirs), _p(coeffs), _p(masks), _p(colors)), self.lib, "ref sh_fwd")

    def _sh_bwd(self, n, K, deg, dirs, coeffs, masks, vcol, cvd, vdirs, vco):
        _check(self.lib.ref_sh_bwd(n, K, deg, _p(dirs), _p(coeffs), _p(masks), _p(vcol), int(cvd),
                                   _p(vdirs), _p(vco)), self.lib, "ref sh_bwd")

    def isect_tile(self, means2d, radii, depths, I, tile_size, tile_width,
                   tile_height, sort=True):
        means2d, radii, depths = _f32(means2d), _i32(radii), _f32(depths)
        N = depths.size // I
        tpg = np.zeros(depths.shape, np.int32)
        m = ct.c_int64()
        _check(self.lib.ref_isect_tile(I, N, _p(means2d), _p(radii), _p(depths), tile_size,
                                       tile_width, tile_height, int(sort), 0, None, None, None,
                                       ct.byref(m)), self.lib, "ref isect_tile")
        ids = np.zeros(m.value, np.int64)
        fids = np.zeros(m.value, np.int32)
        _check(self.lib.ref_isect_tile(I, N, _p(means2d), _p(radii), _p(depths), tile_size,
                                       tile_width, tile_height, int(sort), m.value, _p(tpg),
                                       _p(ids), _p(fids), ct.byref(m)), self.lib, "ref isect_tile")
        return {"tiles_per_gauss": tpg, "isect_ids": ids, "flatten_ids": fids}

    def _isect_offset(self, m, ids, I, tw, th, out):
        _check(self.lib.ref_isect_offset(m, _p(ids), I, tw, th, _p(out)), self.lib, "ref isect_offset")

    def _raster_fwd(self, I, N, ch, m2, con, col, op, bg, masks, W, H, ts, tw, th,
                    toff, m, fids, rc, ra, li, threads=None):
        _check(self.lib.ref_raster_fwd(I, N, ch, _p(m2), _p(con), _p(col), _p(op), _p(bg), _p(masks),
                                       W, H, ts, tw, th, _p(toff), m, _p(fids), _p(rc), _p(ra), _p(li)),
               self.lib, "ref raster_fwd")

    def _raster_bwd(self, I, N, ch, m2, con, col, op, bg, masks, W, H, ts, tw, th,
                    toff, m, fids, ra, li, vrc, vra, absgrad, vabs, vm2, vcon, vcol, vop, vbg,
                    threads=None):
        _check(self.lib.ref_raster_bwd(I, N, ch, _p(m2), _p(con), _p(col), _p(op), _p(bg), _p(masks),
                                       W, H, ts, tw, th, _p(toff), m, _p(fids), _p(ra), _p(li), _p(vrc),
                                       _p(vra), int(absgrad), _p(vabs), _p(vm2), _p(vcon), _p(vcol),
                                       _p(vop), _p(vbg)), self.lib, "ref raster_bwd")


class ReferenceOnDevice(Reference):
    """The reference's front-ends with every node evaluated by the product's
    CUDA eval_gpu adapter (``make -C oracle ref_cuda``): the C++ integration
    path, run on host buffers through the same bridge as ``Reference``."""

    @staticmethod
    def available(path: str = REF_CUDA_SO) -> bool:
        """Built, and against the current C ABI header: a build from an older
        header would pass the library parameter structs of another layout."""
        return os.path.exists(path) and ReferenceOnDevice.abi_current(path)

    @staticmethod
    def abi_current(path: str = REF_CUDA_SO) -> bool:
        import hashlib
        header = os.path.join(os.path.dirname(_HERE), "include", "gsplat_b200.h")
        try:
            with open(path + ".abi") as f:
                built = f.read().strip()
            with open(header, "rb") as f:
                return built == hashlib.sha256(f.read()).hexdigest()
        except OSError:
            return False

    def __init__(self, path: str = REF_CUDA_SO):
        if not self.abi_current(path):
            raise RuntimeError(f"{path} was built against another gsplat_b200.h "
                               "(make -C oracle ref_cuda)")
        super().__init__(path)
        self.lib.ref_b200_sort.argtypes = [_i64, _i, _vp, _vp, _vp, _vp]

    def b200_sort(self, isect_ids, flatten_ids, key_bits):
        """The adapter's one-Primitive stable sort."""
        ids = np.ascontiguousarray(isect_ids, np.int64)
        fids = np.ascontiguousarray(flatten_ids, np.int32)
        out_ids, out_fids = np.zeros_like(ids), np.zeros_like(fids)
        _check(self.lib.ref_b200_sort(ids.size, int(key_bits), _p(ids), _p(fids), _p(out_ids),
                                      _p(out_fids)), self.lib, "adapter sort")
        return out_ids, out_fids
