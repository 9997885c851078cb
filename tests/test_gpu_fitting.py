"""The on-device image-fitting iteration (gsplat_core.fitting: activations,
render, L2 loss, backward, MLX Adam, quaternion renormalisation) against
the same iteration written with torch autograd over the differentiable
operators and a plain torch Adam without bias correction (the trainer's
mlx.optimizers.Adam, scripts/test/train_image_fitting_3dgs_mlx.py:529-566)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _problem(n=3000, size=96, seed=3):
    from gsplat_core import synthetic as S
    sc = S.config2(seed=seed)
    rng = np.random.default_rng(seed)
    idx = np.sort(rng.choice(sc.n, size=n, replace=False))
    K = S.intrinsics(size, size, size / 2, size / 2)
    quats = (sc.quats[idx] * rng.uniform(0.5, 2.0, size=(n, 1))).astype(np.float32)  # not unit
    log_scales = np.log(sc.scales[idx]).astype(np.float32) + 1.5   # larger, so they overlap
    color_logits = rng.normal(size=(n, 3)).astype(np.float32)
    opacity_logits = rng.normal(size=n).astype(np.float32)
    target = S.fitting_target(seed, size, size)
    return (sc.means[idx].copy(), quats, log_scales, color_logits, opacity_logits,
            sc.viewmats[0], K, target, size)


def _torch_step(gs, raw, view, K, target, size, lr=1e-2, b1=0.9, b2=0.999, eps=1e-8, state=None):
    from gsplat_core import autograd as A
    ts = 16
    tw = th = (size + ts - 1) // ts
    ps = [t.clone().requires_grad_(True) for t in raw]
    means, quats, log_scales, color_logits, opacity_logits = ps
    qn = quats / torch.clamp(quats.norm(dim=-1, keepdim=True), min=1e-8)
    m2, dep, con, _, radii = A.projection_ewa_3dgs_fused(
        means[None], view[None], K[None], size, size, quats=qn[None],
        scales=torch.exp(log_scales)[None])
    with torch.no_grad():
        it = gs.intersect_tile_forward({"means2d": m2.detach().view(1, -1, 2),
                                        "radii": radii.view(1, -1, 2),
                                        "depths": dep.detach().view(1, -1)}, 1, ts, tw, th)
        offs = gs.intersect_offset_forward(it["isect_ids"], 1, tw, th)
    rc, _, _ = A.rasterize_to_pixels_3dgs(
        m2.view(1, -1, 2), con.view(1, -1, 3), torch.sigmoid(color_logits)[None],
        torch.sigmoid(opacity_logits)[None], offs, it["flatten_ids"], size, size, ts,
        backgrounds=torch.zeros((1, 3), device="cuda"))
    loss = ((rc - target[None]) ** 2).mean()
    loss.backward()
    if state is None:
        state = [(torch.zeros_like(p), torch.zeros_like(p)) for p in ps]
    out = []
    with torch.no_grad():
        for p, (m, v) in zip(ps, state):
            m.mul_(b1).add_((1 - b1) * p.grad)
            v.mul_(b2).add_((1 - b2) * p.grad * p.grad)
            out.append(p - lr * m / (torch.sqrt(v) + eps))
        out[1] = out[1] / torch.clamp(out[1].norm(dim=-1, keepdim=True), min=1e-8)
    return [o.detach() for o in out], float(loss), state


def test_fit_iteration_matches_torch(gs, cuda):
    from gsplat_core import fitting
    means, quats, log_scales, cl, ol, view, K, target, size = _problem()
    T = lambda x: torch.from_numpy(np.ascontiguousarray(x)).cuda()  # noqa: E731
    fit = fitting.ImageFitStep(means, quats, log_scales, cl, ol, view, K, target, size, size)
    raw = [T(means), T(quats), T(log_scales), T(cl), T(ol)]
    state = None
    for it in range(3):
        loss = float(fit.run().item())
        raw, loss_ref, state = _torch_step(gs, raw, T(view), T(K), T(target), size, state=state)
        assert abs(loss - loss_ref) <= 1e-5 * max(1.0, abs(loss_ref)), (it, loss, loss_ref)
        # Adam's first steps move each parameter by about lr * sign(g); a
        # different atomic order only matters where g is near zero
        for name, a, b in zip(("means", "quats", "log_scales", "color_logits", "opacity_logits"),
                              (fit.means, fit.quats, fit.log_scales, fit.color_logits,
                               fit.opacity_logits), raw):
            d = (a.reshape(b.shape) - b).abs()
            bad = (d > 2e-3).float().mean().item()
            assert bad < 2e-3, f"step {it} {name}: {bad:.2%} of entries differ (max {d.max():.3g})"


def test_fit_descends(gs, cuda):
    from gsplat_core import fitting
    means, quats, log_scales, cl, ol, view, K, target, size = _problem(n=3000, size=96, seed=5)
    fit = fitting.ImageFitStep(means, quats, log_scales, cl, ol, view, K, target, size, size)
    losses = [float(fit.run().item()) for _ in range(60)]
    assert all(np.isfinite(losses))
    assert losses[-1] < 0.7 * losses[0], losses[::10]
    q = fit.quats
    assert torch.allclose(q.norm(dim=-1), torch.ones_like(q[:, 0]), atol=1e-5)
