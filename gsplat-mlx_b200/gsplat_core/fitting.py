"""On-device iteration of the reference's image-fitting trainer
(scripts/test/train_image_fitting_3dgs_mlx.py): raw parameters (means,
quats, log_scales, color_logits, opacity_logits), their activations
(:33-36, :104-118), render + L2 loss + backward through the native
operators, and MLX Adam (defaults: betas 0.9 / 0.999, eps 1e-8, no bias
correction; lr 1e-2 for every group, :378-382 and :529-566) with the
trainer's quaternion renormalisation -- every stage a kernel of
libgsplat_b200.so, one host read per step (the intersection count), plus
the loss when the caller reads it (the trainer prints it every step).
"""
from __future__ import annotations

import ctypes as ct

import torch

from . import _lib
from ._lib import AdamParams, check
from .pipeline import TrainingStep, _p, _s


class ImageFitStep:
    def __init__(self, means, quats, log_scales, color_logits, opacity_logits, viewmat, K,
                 target, width, height, lr=1.0e-2, beta1=0.9, beta2=0.999, eps=1.0e-8,
                 tile_size=16, far_plane=1.0e10, device=None):
        self.dev = device or torch.device("cuda", torch.cuda.current_device())
        f = lambda x: torch.as_tensor(x, dtype=torch.float32).to(self.dev).contiguous()  # noqa
        self.means, self.quats = f(means).clone(), f(quats).clone()
        self.log_scales, self.color_logits = f(log_scales).clone(), f(color_logits).clone()
        self.opacity_logits = f(opacity_logits).clone().reshape(-1)
        self.viewmats, self.Ks = f(viewmat).reshape(1, 4, 4), f(K).reshape(1, 3, 3)
        self.target = f(target).reshape(1, height, width, 3)
        n = self.means.shape[0]
        self.n = n
        self.lib = _lib.load()
        e = lambda *shape: torch.empty(shape, dtype=torch.float32, device=self.dev)  # noqa: E731
        self.quats_n, self.scales, self.colors, self.opacities = e(n, 4), e(n, 3), e(n, 3), e(n)
        self.m1 = torch.zeros((n, 14), dtype=torch.float32, device=self.dev)
        self.m2 = torch.zeros((n, 14), dtype=torch.float32, device=self.dev)
        self.hp = AdamParams(n, float(lr), float(beta1), float(beta2), float(eps))
        self.step = TrainingStep(n, 0, 1, 1, width, height, tile_size=tile_size,
                                 far_plane=far_plane, device=self.dev)
        self.coeffs_unused = e(n, 1, 3)
        check(self.lib.gs_fit_activate(n, _p(self.quats), _p(self.log_scales),
                                       _p(self.color_logits), _p(self.opacity_logits),
                                       _p(self.quats_n), _p(self.scales), _p(self.colors),
                                       _p(self.opacities), _s()), "fit_activate")

    def run(self):
        """One training iteration; returns the device scalar holding this
        step's loss (evaluated before the update, as the trainer reports)."""
        st = self.step
        st.run(self.means, self.quats_n, self.scales, self.opacities, self.coeffs_unused,
               self.viewmats, self.Ks, None, None, colors=self.colors, target=self.target)
        check(self.lib.gs_fit_adam(ct.byref(self.hp), _p(self.means), _p(self.quats),
                                   _p(self.log_scales), _p(self.color_logits),
                                   _p(self.opacity_logits), _p(st.v_means), _p(st.v_quats),
                                   _p(st.v_scales), _p(st.v_colors), _p(st.v_opacities),
                                   _p(self.m1), _p(self.m2), _p(self.quats_n), _p(self.scales),
                                   _p(self.colors), _p(self.opacities), _s()), "fit_adam")
        st._mark("adam")
        return st.loss
