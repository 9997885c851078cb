"""Densification statistics of the reference trainer's default strategy on
device (scripts/test/scanner_points_training_utils.py,
ScannerDefaultStrategyRuntime, :355-889): the per-step grad2d / count /
2D-radius accumulation of update_state and the clone / split / prune masks
of a refine step, as kernels of libgsplat_b200.so (gs_densify_accumulate,
gs_densify_masks).  The statistics match the reference bit for bit; the
masks match except where a scale or opacity lies within a few ulp of its
threshold (expf against numpy's exp).

The topology edits that follow a refine (gathering, appending and dropping
parameter and optimizer rows every refine_every steps) are the caller's:
``apply_keep`` / ``apply_duplicate`` / ``apply_split`` keep these statistics
in step with them the way the reference's _apply_*_to_state do.
"""
from __future__ import annotations

import ctypes as ct
from dataclasses import dataclass

import torch

from . import _lib
from ._lib import DensifyMaskParams, DensifyParams, check


@dataclass
class DensifyConfig:
    """ScannerDefaultStrategyConfig's thresholds and schedule (:324-353)."""
    prune_opa: float = 0.005
    grow_grad2d: float = 0.0002
    grow_scale3d: float = 0.01
    grow_scale2d: float = 0.05
    prune_scale3d: float = 0.1
    prune_scale2d: float = 0.15
    refine_scale2d_stop_iter: int = 0
    refine_start_iter: int = 500
    refine_stop_iter: int = 15000
    reset_every: int = 3000
    refine_every: int = 100
    pause_refine_after_reset: int = 0
    scene_scale: float = 1.0

    def should_refine(self, step: int) -> bool:
        return (self.refine_start_iter < step < self.refine_stop_iter
                and step % self.refine_every == 0
                and step % self.reset_every >= self.pause_refine_after_reset)

    def should_reset_opacity(self, step: int) -> bool:
        return step > 0 and step % self.reset_every == 0


def _p(t):
    return None if t is None else ct.c_void_p(t.data_ptr())


def _s():
    return ct.c_void_p(torch.cuda.current_stream().cuda_stream)


class DensifyStats:
    """grad2d, count and (when the config tracks 2D radii) the running max
    of the normalised radii, one float per Gaussian, on device."""

    def __init__(self, n: int, config: DensifyConfig | None = None, device=None):
        self.config = config or DensifyConfig()
        self.dev = device or torch.device("cuda", torch.cuda.current_device())
        self.lib = _lib.load()
        self.totals = torch.zeros((6,), dtype=torch.int64, device=self.dev)
        self.reset(n)

    @property
    def track_radii(self) -> bool:
        return self.config.refine_scale2d_stop_iter > 0

    def reset(self, n: int) -> None:
        """reset_running_state (:397-404)."""
        z = lambda: torch.zeros((int(n),), dtype=torch.float32, device=self.dev)  # noqa: E731
        self.grad2d, self.count = z(), z()
        self.radii = z() if self.track_radii else None

    def update_state(self, v_means2d, radii, width: int, height: int, n_cameras: int) -> None:
        """update_state (:412-451) for [C, N, 2] (or [N, 2]) screen-space
        mean gradients -- or their absgrad -- and radii of one step."""
        v = v_means2d.reshape(-1, self.grad2d.numel(), 2).contiguous()
        r = radii.reshape(-1, self.grad2d.numel(), 2).to(torch.int32).contiguous()
        p = DensifyParams(v.shape[0], self.grad2d.numel(), int(width), int(height), int(n_cameras))
        check(self.lib.gs_densify_accumulate(ct.byref(p), _p(v), _p(r), _p(self.grad2d),
                                             _p(self.count), _p(self.radii), _s()),
              "densify_accumulate")

    def masks(self, step: int, log_scales, opacity_logits, n_original: int | None = None,
              grow: bool = True, prune: bool = True):
        """Boolean clone / split masks (grow) over the statistics' Gaussians
        and the prune mask over ``log_scales``' Gaussians, with counts:
        {"clone", "split", "prune", "n_clone", "n_split", "prune_breakdown"}.
        The reference takes clone and split before either is applied and
        prune after both (call with grow=False, prune=True then)."""
        c = self.config
        n = log_scales.shape[-2] if log_scales.dim() > 1 else log_scales.numel() // 3
        ls = log_scales.reshape(n, 3).contiguous()
        ol = opacity_logits.reshape(n).contiguous() if opacity_logits is not None else None
        u8 = lambda: torch.empty((n,), dtype=torch.uint8, device=self.dev)  # noqa: E731
        clone, split, prn = (u8() if grow else None), (u8() if grow else None), (u8() if prune else None)
        p = DensifyMaskParams(n, n if n_original is None else int(n_original), int(step), int(grow),
                              int(prune), int(c.refine_scale2d_stop_iter), int(c.reset_every), 0,
                              c.grow_grad2d, c.grow_scale3d, c.grow_scale2d, c.prune_opa,
                              c.prune_scale3d, c.prune_scale2d, c.scene_scale)
        check(self.lib.gs_densify_masks(ct.byref(p), _p(self.grad2d), _p(self.count),
                                        _p(self.radii), _p(ls), _p(ol), _p(clone), _p(split),
                                        _p(prn), _p(self.totals), _s()), "densify_masks")
        t = self.totals.tolist()
        out = {}
        if grow:
            out.update(clone=clone.bool(), split=split.bool(), n_clone=t[0], n_split=t[1])
        if prune:
            out.update(prune=prn.bool(), prune_breakdown=t[3:6] + [t[2]])
        return out

    def stats(self) -> dict:
        """_grad2d_stats (:453-465)."""
        vis = self.count > 0
        avg = torch.where(vis, self.grad2d / torch.clamp(self.count, min=1.0),
                          torch.zeros_like(self.grad2d))
        nv = int(vis.sum())
        return {"visible_gaussians": nv, "total_observations": int(self.count.sum()),
                "grad2d_mean": float(avg[vis].mean()) if nv else 0.0,
                "grad2d_max": float(avg[vis].max()) if nv else 0.0,
                "count_max": float(self.count.max()) if self.count.numel() else 0.0,
                "radii_max": (float(self.radii.max()) if self.radii is not None
                              and self.radii.numel() else None)}

    def _each(self):
        return [a for a in (self.grad2d, self.count, self.radii) if a is not None]

    def _set(self, arrays):
        self.grad2d, self.count = arrays[0], arrays[1]
        if self.radii is not None:
            self.radii = arrays[2]

    def apply_keep(self, keep_idx) -> None:
        """_apply_keep_to_state (:467-472)."""
        self._set([a[keep_idx] for a in self._each()])

    def apply_duplicate(self, selected_idx) -> None:
        """_apply_duplicate_to_state (:497-502): selected rows appended."""
        self._set([torch.cat([a, a[selected_idx]]) for a in self._each()])

    def apply_split(self, split_mask) -> None:
        """_apply_split_to_state (:586-592): unsplit rows, then the split
        rows twice."""
        rest, sel = ~split_mask, split_mask
        self._set([torch.cat([a[rest], a[sel], a[sel]]) for a in self._each()])
