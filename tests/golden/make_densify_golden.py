"""Generate tests/golden/densify.npz from the reference trainer's own
densification runtime (scripts/test/scanner_points_training_utils.py,
ScannerDefaultStrategyRuntime), run in this container.

That module imports MLX, the reference's nanobind gsplat_core and two
dataset helpers, none of which the strategy's numpy bookkeeping needs; they
are replaced by stand-ins (MLX's array calls map to their numpy
equivalents, the rest are unused names) so that the reference's own class
runs unchanged on numpy arrays.  Recorded: the grad2d / count / radius
statistics after several update_state calls, the clone selection, the split
mask, and the prune inputs, breakdown and keep set of one refine step, plus
every input.

    python tests/golden/make_densify_golden.py [path to the reference's scripts/test]
"""
from __future__ import annotations

import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _install_stand_ins():
    mx = types.ModuleType("mlx.core")
    mx.float32, mx.int32 = np.float32, np.int32
    mx.eval = lambda *a, **k: None
    mx.array = lambda x, dtype=None: np.asarray(x, dtype=dtype)
    mx.take = lambda a, idx, axis=None: np.take(a, np.asarray(idx), axis=axis)
    mx.concatenate = lambda xs, axis=0: np.concatenate(xs, axis=axis)
    mx.zeros_like = np.zeros_like
    mx.minimum = np.minimum
    mx.sqrt, mx.sum = np.sqrt, np.sum
    nn = types.ModuleType("mlx.nn")
    nn.Module = object
    opt = types.ModuleType("mlx.optimizers")
    opt.Adam = object
    mlx = types.ModuleType("mlx")
    mlx.core, mlx.nn, mlx.optimizers = mx, nn, opt
    gs = types.ModuleType("gsplat_core")
    for name in ("intersect_offset_forward", "intersect_tile_forward",
                 "projection_ewa_3dgs_fused_forward", "rasterize_to_pixels_3dgs_forward",
                 "spherical_harmonics_forward"):
        setattr(gs, name, None)
    png = types.ModuleType("render_random_3dgs_png")
    png.write_png = None
    ds = types.ModuleType("scanner_dataset_utils")
    for name in ("axis_transform", "collect_frames", "load_camera", "load_target"):
        setattr(ds, name, None)
    sys.modules.update({"mlx": mlx, "mlx.core": mx, "mlx.nn": nn, "mlx.optimizers": opt,
                        "gsplat_core": gs, "render_random_3dgs_png": png,
                        "scanner_dataset_utils": ds})


class _Model:
    """The attributes the strategy reads and replaces (reference layout:
    a leading batch axis, GAUSSIAN_AXES)."""

    def __init__(self, means, quats, log_scales, opacity_logits, color_logits):
        self.means, self.quats, self.log_scales = means[None], quats[None], log_scales[None]
        self.opacity_logits, self.color_logits = opacity_logits[None], color_logits[None, None]

    @property
    def normalized_quats(self):
        q = self.quats
        return q / np.maximum(np.sqrt(np.sum(q * q, axis=-1, keepdims=True)), 1e-8)


def main(ref_dir):
    _install_stand_ins()
    sys.path.insert(0, ref_dir)
    import scanner_points_training_utils as R  # the reference module, unchanged

    rng = np.random.default_rng(77)
    C, N, W, H = 3, 3000, 256, 192
    T = 4  # update_state calls
    v_means2d = (rng.standard_normal((T, C, N, 2)) * 4.0e-7).astype(np.float32)
    radii = rng.integers(0, 10, size=(T, C, N, 2)).astype(np.int32)
    big = rng.uniform(size=(T, C, N)) < 0.03
    radii[big] = rng.integers(10, 40, size=(int(big.sum()), 2))
    radii[rng.uniform(size=(T, C, N)) < 0.3] = 0
    means = rng.uniform(-1, 1, size=(N, 3)).astype(np.float32)
    quats = rng.standard_normal((N, 4)).astype(np.float32)
    log_scales = rng.uniform(-6.0, -1.8, size=(N, 3)).astype(np.float32)
    opacity_logits = rng.uniform(-7.0, 3.0, size=(N,)).astype(np.float32)
    color_logits = rng.standard_normal((N, 3)).astype(np.float32)
    cfg = R.ScannerDefaultStrategyConfig(enabled=True, refine_scale2d_stop_iter=5000)
    step = 3100  # refines, past reset_every: every prune reason is live
    rt = R.ScannerDefaultStrategyRuntime(cfg, N)
    for t in range(T):
        # a copy: with numpy inputs np.asarray does not copy and update_state
        # scales its argument in place (an MLX array is copied out first)
        rt.update_state(v_means2d[t].copy(), radii[t], W, H, C)
    stats = {"grad2d": rt.grad2d.copy(), "count": rt.count.copy(), "radii": rt.radii.copy()}

    rec = {}
    orig_dup = rt._apply_duplicate_to_state
    orig_split = rt._apply_split_to_state
    orig_prune = rt._prune_gaussians
    orig_keep = rt._apply_keep_to_state

    def dup(selected):
        rec["clone_selected"] = np.asarray(selected, np.int64)
        return orig_dup(selected)

    def split(mask):
        rec["split_mask"] = np.asarray(mask, bool)
        return orig_split(mask)

    def prune(step_, model, optimizers, color_mode):
        rec["prune_log_scales"] = np.asarray(model.log_scales[0], np.float32).copy()
        rec["prune_opacity_logits"] = np.asarray(model.opacity_logits[0], np.float32).copy()
        rec["prune_radii"] = rt.radii.copy()
        n, breakdown = orig_prune(step_, model, optimizers, color_mode)
        rec["prune_breakdown"] = np.array([breakdown["opacity"], breakdown["scale3d"],
                                           breakdown["scale2d"], breakdown["total_unique"]],
                                          np.int64)
        return n, breakdown

    def keep(k):
        rec["prune_keep"] = np.asarray(k, np.int64)
        return orig_keep(k)

    rt._apply_keep_to_state = keep
    rt._apply_duplicate_to_state = dup
    rt._apply_split_to_state = split
    rt._prune_gaussians = prune
    model = _Model(means, quats, log_scales, opacity_logits, color_logits)
    rt.after_optimizer_step(step, model, {}, "rgb")
    out = dict(C=C, N=N, W=W, H=H, step=step, v_means2d=v_means2d, radii_in=radii,
               log_scales=log_scales, opacity_logits=opacity_logits,
               grow_grad2d=cfg.grow_grad2d, grow_scale3d=cfg.grow_scale3d,
               grow_scale2d=cfg.grow_scale2d, prune_opa=cfg.prune_opa,
               prune_scale3d=cfg.prune_scale3d, prune_scale2d=cfg.prune_scale2d,
               scene_scale=cfg.scene_scale, refine_scale2d_stop_iter=cfg.refine_scale2d_stop_iter,
               reset_every=cfg.reset_every, **stats)
    out.update(rec)
    out.setdefault("clone_selected", np.zeros((0,), np.int64))
    out.setdefault("split_mask", np.zeros((N,), bool))
    np.savez_compressed(os.path.join(HERE, "densify.npz"), **out)
    print({k: (v.shape if hasattr(v, "shape") else v) for k, v in out.items()})


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else
         os.path.join(os.sep, "root", "reference", "scripts", "test"))
