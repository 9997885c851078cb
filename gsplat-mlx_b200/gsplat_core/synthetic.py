"""Seeded synthetic scenes with the shapes and value distributions of the
five benchmark configurations the reference's hot path is measured on.

No public dataset is involved: every array comes from
``numpy.random.default_rng(seed)``.  Activations are applied the way the
reference trainers apply them before calling the operators
(scripts/test/scanner_points_training_utils.py:306-316): scales =
exp(log-scales), opacities = sigmoid(logits), quaternions normalised.

Cameras follow the reference's convention: ``viewmats`` are world-to-camera
4x4 row-major matrices with x right, y down, z forward
(gsplat_projection.cpp:483-493), ``Ks`` are pinhole intrinsics.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np


@dataclass
class Scene:
    name: str
    means: np.ndarray          # [N, 3]
    quats: np.ndarray          # [N, 4] (w, x, y, z), unit
    scales: np.ndarray         # [N, 3]
    opacities: np.ndarray      # [N]
    sh_degree: int
    coeffs: np.ndarray         # [N, K, 3] with K = (sh_degree + 1)^2
    colors: np.ndarray | None  # [N, 3] for SH degree 0 configs fed directly
    viewmats: np.ndarray       # [C, 4, 4]
    Ks: np.ndarray             # [C, 3, 3]
    width: int
    height: int
    tile_size: int = 16
    eps2d: float = 0.3
    near_plane: float = 0.01
    far_plane: float = 1e10
    background: np.ndarray = field(default_factory=lambda: np.zeros(3, np.float32))
    seed: int = 0

    @property
    def n(self) -> int:
        return int(self.means.shape[0])

    @property
    def cameras(self) -> int:
        return int(self.viewmats.shape[0])

    @property
    def tile_width(self) -> int:
        return (self.width + self.tile_size - 1) // self.tile_size

    @property
    def tile_height(self) -> int:
        return (self.height + self.tile_size - 1) // self.tile_size


def look_at(position, target=(0.0, 0.0, 0.0)) -> np.ndarray:
    """World-to-camera matrix for a camera at ``position`` facing ``target``
    (x right, y down, z forward; world +y is "down")."""
    p = np.asarray(position, np.float64)
    f = np.asarray(target, np.float64) - p
    f /= np.linalg.norm(f)
    down0 = np.array([0.0, 1.0, 0.0])
    right = np.cross(down0, f)
    if np.linalg.norm(right) < 1e-8:
        right = np.array([1.0, 0.0, 0.0])
    right /= np.linalg.norm(right)
    down = np.cross(f, right)
    R = np.stack([right, down, f], axis=0)
    M = np.eye(4)
    M[:3, :3] = R
    M[:3, 3] = -R @ p
    return M.astype(np.float32)


def intrinsics(fx, fy, cx, cy) -> np.ndarray:
    return np.array([[fx, 0.0, cx], [0.0, fy, cy], [0.0, 0.0, 1.0]], np.float32)


def orbit(count, radius, elevation=0.25):
    """``count`` look-at cameras evenly spaced on a circle of ``radius``
    around the origin, raised by ``elevation * radius``."""
    mats = []
    for c in range(count):
        th = 2.0 * np.pi * c / count
        mats.append(look_at((radius * np.sin(th), -elevation * radius, radius * np.cos(th))))
    return np.stack(mats, 0)


def _unit_quats(rng, n):
    q = rng.normal(size=(n, 4)).astype(np.float32)
    q /= np.linalg.norm(q, axis=1, keepdims=True)
    return q.astype(np.float32)


def _sigmoid(x):
    return (1.0 / (1.0 + np.exp(-x))).astype(np.float32)


def _sh_coeffs(rng, n, degree):
    K = (degree + 1) ** 2
    co = np.empty((n, K, 3), np.float32)
    co[:, 0, :] = rng.uniform(0.0, 1.0, size=(n, 3))
    if K > 1:
        co[:, 1:, :] = rng.normal(0.0, 0.05, size=(n, K - 1, 3))
    return co


def _clustered_means(rng, n, clusters=64, half_box=5.0):
    centres = rng.uniform(-0.8 * half_box, 0.8 * half_box, size=(clusters, 3))
    axes = rng.uniform(0.1, 1.0, size=(clusters, 3))
    rots = []
    for _ in range(clusters):
        a, _ = np.linalg.qr(rng.normal(size=(3, 3)))
        rots.append(a)
    rots = np.stack(rots, 0)
    which = rng.integers(0, clusters, size=n)
    local = rng.normal(size=(n, 3)) * axes[which]
    pts = centres[which] + np.einsum("nij,nj->ni", rots[which], local)
    return np.clip(pts, -half_box, half_box).astype(np.float32)


def config1(seed=0) -> Scene:
    """N=10k random Gaussians, SH0 colours fed straight to rasterize, one
    256x256 camera at (0,0,-3) looking down +z (benchmark config 1)."""
    rng = np.random.default_rng(seed)
    n = 10_000
    means = rng.uniform(-1.0, 1.0, size=(n, 3)).astype(np.float32)
    quats = _unit_quats(rng, n)
    scales = np.exp(rng.uniform(-5.0, -3.0, size=(n, 3))).astype(np.float32)
    opac = _sigmoid(rng.normal(size=n))
    colors = rng.uniform(0.0, 1.0, size=(n, 3)).astype(np.float32)
    view = np.eye(4, dtype=np.float32)
    view[2, 3] = 3.0
    return Scene("cfg1", means, quats, scales, opac, 0, colors[:, None, :].copy(), colors,
                 view[None], intrinsics(256, 256, 128, 128)[None], 256, 256, seed=seed)


def config2(seed=0) -> Scene:
    """N=100k near-planar Gaussians for 2D image fitting at 512x512
    (benchmark config 2)."""
    rng = np.random.default_rng(seed)
    n = 100_000
    means = np.empty((n, 3), np.float32)
    means[:, :2] = rng.uniform(-1.0, 1.0, size=(n, 2))
    means[:, 2] = rng.uniform(-0.01, 0.01, size=n)
    quats = _unit_quats(rng, n)
    scales = np.exp(rng.uniform(-5.0, -3.0, size=(n, 3))).astype(np.float32)
    opac = _sigmoid(rng.normal(size=n))
    colors = rng.uniform(0.0, 1.0, size=(n, 3)).astype(np.float32)
    view = np.eye(4, dtype=np.float32)
    view[2, 3] = 8.0
    return Scene("cfg2", means, quats, scales, opac, 0, colors[:, None, :].copy(), colors,
                 view[None], intrinsics(512, 512, 256, 256)[None], 512, 512, seed=seed)


def fitting_target(seed=0, width=512, height=512, waves=8) -> np.ndarray:
    """Smooth RGB target in [0, 1]: a sum of ``waves`` random 2D sinusoids."""
    rng = np.random.default_rng(seed + 1000)
    yy, xx = np.meshgrid(np.linspace(0, 1, height), np.linspace(0, 1, width), indexing="ij")
    img = np.zeros((height, width, 3))
    for _ in range(waves):
        k = rng.uniform(1.0, 8.0, size=2) * 2 * np.pi
        ph = rng.uniform(0, 2 * np.pi)
        amp = rng.uniform(0.2, 1.0, size=3)
        img += amp * np.sin(k[0] * xx + k[1] * yy + ph)[..., None]
    img -= img.min()
    img /= max(img.max(), 1e-8)
    return img.astype(np.float32)


def _scene_sh3(name, rng, n, log_scale_range, viewmats, K, width, height, seed):
    means = _clustered_means(rng, n)
    quats = _unit_quats(rng, n)
    scales = np.exp(rng.uniform(*log_scale_range, size=(n, 3))).astype(np.float32)
    opac = _sigmoid(rng.normal(size=n))
    coeffs = _sh_coeffs(rng, n, 3)
    C = viewmats.shape[0]
    Ks = np.repeat(K[None], C, axis=0)
    return Scene(name, means, quats, scales, opac, 3, coeffs, None, viewmats, Ks,
                 width, height, seed=seed)


def config3(seed=0, n=1_000_000) -> Scene:
    """N=1M SH3 Gaussians in 64 anisotropic clusters inside a 10 m box; one
    1297x840 camera (fx=fy=1150) 4 m from the box centre facing it
    (benchmark config 3, the single-GPU headline)."""
    rng = np.random.default_rng(seed)
    view = look_at((0.0, -1.0, -3.87298))[None]  # |p| = 4 m
    return _scene_sh3("cfg3", rng, n, (-6.0, -2.0), view,
                      intrinsics(1150, 1150, 648.5, 420.0), 1297, 840, seed)


def config4(seed=0, n=3_000_000, cameras=32) -> Scene:
    """N=3M SH3 Gaussians, 32 cameras 1920x1080 (fx=fy=1600) on a 5 m
    orbit (benchmark config 4, camera-sharded multi-GPU step)."""
    rng = np.random.default_rng(seed)
    return _scene_sh3("cfg4", rng, n, (-6.0, -2.0), orbit(cameras, 5.0),
                      intrinsics(1600, 1600, 960.0, 540.0), 1920, 1080, seed)


def config5(seed=0, n=6_000_000, cameras=8) -> Scene:
    """N=6M SH3 Gaussians with log-scales U[-3,-1] (heavy overdraw), 8
    cameras 3840x2160 (fx=fy=3000) on a 3 m orbit (benchmark config 5)."""
    rng = np.random.default_rng(seed)
    return _scene_sh3("cfg5", rng, n, (-3.0, -1.0), orbit(cameras, 3.0),
                      intrinsics(3000, 3000, 1920.0, 1080.0), 3840, 2160, seed)


CONFIGS = {"cfg1": config1, "cfg2": config2, "cfg3": config3, "cfg4": config4, "cfg5": config5}


def cotangents(seed, images, height, width, channels=3):
    """Backward drivers of the benchmark: dL/dcolor ~ N(0,1), dL/dalpha ~ N(0,0.1)."""
    rng = np.random.default_rng(seed + 7)
    v_colors = rng.normal(0.0, 1.0, size=(images, height, width, channels)).astype(np.float32)
    v_alphas = rng.normal(0.0, 0.1, size=(images, height, width, 1)).astype(np.float32)
    return v_colors, v_alphas
