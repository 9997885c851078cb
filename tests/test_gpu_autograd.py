"""Reverse-mode wiring (gsplat_core.autograd), the counterpart of the
reference Primitives' vjp methods and of its autograd smokes
(scripts/test/autograd_vjp_smoke.py, training_dense_3dgs_loop_smoke.py,
training_projection_viewspace_proxy_smoke.py)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from _util import assert_grad_close

pytestmark = pytest.mark.gpu


def T(x, grad=False):
    t = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    return t.requires_grad_(grad)


def _render(gs, A, means, quats, scales, opac, coeffs, view, K, W, H, vsp=None, bg=None):
    """The trainers' render_sh_model (scanner_points_training_utils.py:
    1050-1122) written with the differentiable operators and torch glue."""
    ts = 16
    tw, th = (W + ts - 1) // ts, (H + ts - 1) // ts
    m2, dep, con, _, radii = A.projection_ewa_3dgs_fused(
        means[None], view[None], K[None], W, H, quats=quats[None], scales=scales[None],
        viewspace_points=vsp)
    with torch.no_grad():
        it = gs.intersect_tile_forward({"means2d": m2.detach().view(1, -1, 2),
                                        "radii": radii.view(1, -1, 2),
                                        "depths": dep.detach().view(1, -1)}, 1, ts, tw, th)
        offs = gs.intersect_offset_forward(it["isect_ids"], 1, tw, th)
    campos = -(view[:3, :3].T @ view[:3, 3])
    d = means - campos
    d = d / torch.clamp(torch.linalg.norm(d, dim=-1, keepdim=True), min=1e-8)
    col = A.spherical_harmonics(3 if coeffs.shape[1] == 16 else 0, d, coeffs)
    col = torch.clamp(col + 0.5, 0.0, 1.0)
    rc, ra, _ = A.rasterize_to_pixels_3dgs(m2.view(1, -1, 2), con.view(1, -1, 3), col[None],
                                           opac[None], offs, it["flatten_ids"], W, H, ts,
                                           backgrounds=bg)
    return rc, ra


def test_autograd_chain_matches_training_step(gs, cuda):
    """Gradients from torch autograd through the operators equal the fused
    training step's (which is parity-tested against the oracle)."""
    from gsplat_core import autograd as A, pipeline, synthetic as S
    sc = S.config3(seed=2, n=40_000)
    sc.Ks = sc.Ks.copy()
    sc.Ks[:, :2, :] /= 2
    W, H = sc.width // 2, sc.height // 2
    vrc, vra = S.cotangents(4, 1, H, W)
    p = [T(sc.means, True), T(sc.quats, True), T(sc.scales, True), T(sc.opacities, True),
         T(sc.coeffs, True)]
    vsp = torch.zeros((1, 1, sc.n, 2), device=cuda, requires_grad=True)
    rc, ra = _render(gs, A, *p, T(sc.viewmats[0]), T(sc.Ks[0]), W, H, vsp=vsp,
                     bg=torch.zeros((1, 3), device=cuda))
    loss = (rc * T(vrc)).sum() + (ra * T(vra)).sum()
    loss.backward()
    step = pipeline.TrainingStep(sc.n, 3, 16, 1, W, H)
    step.run(*[x.detach() for x in p], T(sc.viewmats), T(sc.Ks), T(vrc), T(vra))
    torch.cuda.synchronize()
    g = step.gradients()
    for name, t in zip(("v_means", "v_quats", "v_scales", "v_opacities", "v_coeffs"), p):
        # two GPU runs differ only by atomic order; heavy cancellation in a
        # few entries needs the wider absolute floor
        assert_grad_close(t.grad, g[name], "autograd " + name, atol_frac=5e-4)
    # viewspace_points receives the means2d cotangent unchanged (cpp:1200-1201)
    assert_grad_close(vsp.grad.view(-1, 2), step.v_means2d.view(-1, 2), "viewspace proxy",
                      atol_frac=1e-6)


def test_autograd_quat_scale_and_viewmats(gs, cuda):
    from gsplat_core import autograd as A
    rng = np.random.default_rng(5)
    q = T(rng.normal(size=(500, 4)).astype(np.float32), True)
    s = T(np.exp(rng.uniform(-2, 0, size=(500, 3))).astype(np.float32), True)
    cov, pre = A.quat_scale_to_covar_preci(q, s)
    w1 = torch.randn_like(cov)
    w2 = torch.randn_like(pre)
    ((cov * w1).sum() + (pre * w2).sum()).backward()
    b = gs.quat_scale_to_covar_preci_backward({"quats": q.detach(), "scales": s.detach()},
                                              {"v_covars": w1, "v_precis": w2})
    assert_grad_close(q.grad, b["v_quats"], "v_quats")
    assert_grad_close(s.grad, b["v_scales"], "v_scales")
    # viewmats gradient only when viewmats requires grad
    from gsplat_core import synthetic as S
    sc = S.config1()
    means = T(sc.means[:2000], True)
    view = T(sc.viewmats[None], True)
    m2, dep, con, _, radii = A.projection_ewa_3dgs_fused(
        means[None], view, T(sc.Ks[None]), sc.width, sc.height, quats=T(sc.quats[:2000][None]),
        scales=T(sc.scales[:2000][None]))
    (m2.sum() + dep.sum() + 1e-3 * con.sum()).backward()
    assert view.grad is not None and torch.isfinite(view.grad).all()
    assert float(view.grad.abs().sum()) > 0
    assert torch.isfinite(means.grad).all()


def test_training_descent_smoke(gs, cuda):
    """A few Gaussians fitted to a target image for 8 Adam steps: the loss
    must not rise more than 5% and every parameter gradient is non-zero
    (mirrors scripts/test/training_dense_3dgs_loop_smoke.py:234-291)."""
    from gsplat_core import autograd as A
    torch.manual_seed(0)
    W = H = 32
    K = torch.tensor([[32.0, 0, 16], [0, 32.0, 16], [0, 0, 1]], device=cuda)
    view = torch.eye(4, device=cuda)
    view[2, 3] = 3.0
    tgt_means = torch.tensor([[-0.4, -0.3, 0.0], [0.4, 0.2, 0.1], [0.0, 0.4, -0.1],
                              [-0.2, 0.3, 0.2]], device=cuda)
    n = tgt_means.shape[0]
    def params(means, seed):
        g = torch.Generator(device="cpu").manual_seed(seed)
        return [means.clone().requires_grad_(True),
                torch.randn(n, 4, generator=g).cuda().requires_grad_(True),
                torch.full((n, 3), -2.0, device=cuda).requires_grad_(True),
                torch.zeros(n, device=cuda).requires_grad_(True),
                (0.3 * torch.randn(n, 1, 3, generator=g)).cuda().requires_grad_(True)]

    def render(ps):
        means, q, log_s, logit, co = ps
        qn = q / q.norm(dim=-1, keepdim=True)
        rc, ra = _render(gs, A, means, qn, torch.exp(log_s), torch.sigmoid(logit), co, view, K,
                         W, H)
        return rc

    with torch.no_grad():
        target = render(params(tgt_means, 1))
    ps = params(tgt_means + 0.08 * torch.randn_like(tgt_means), 2)
    opt = torch.optim.Adam(ps, lr=0.01)
    losses = []
    for _ in range(8):
        opt.zero_grad()
        loss = ((render(ps) - target) ** 2).mean()
        loss.backward()
        losses.append(float(loss))
        for p_ in ps:
            assert p_.grad is not None and float(p_.grad.abs().sum()) > 0
        opt.step()
    assert losses[-1] <= losses[0] * 1.05, losses
