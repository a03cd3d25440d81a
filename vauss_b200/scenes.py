"""Seeded synthetic splat scenes and cameras for the benchmark configurations.

The reference quotes its numbers on public capture datasets that are not
available here; these generators stand in for them with the shapes, sizes and
value distributions the benchmark configurations name.  Parameters use the
reference's per-splat layout (crates/splat-train-render/src/gaussian_splats.rs:
131-153): ``transforms [N, 10]`` = mean (3), quaternion (w, x, y, z) (4),
log-scale (3); ``sh_coeffs [N, (d+1)^2, 3]``; ``raw_opacities [N]`` (logits).

SH DC values are drawn as RGB colours and stored as coefficients through the
reference's ``rgb_to_sh`` (crates/splat-train-render/src/sh.rs:21-31:
``(rgb - 0.5) / SH_C0``), so the rendered base colour is the drawn colour.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .camera import Camera, look_at

SH_C0 = np.float32(0.2820948)


@dataclass
class SplatSet:
    transforms: np.ndarray  # [N, 10] f32
    sh: np.ndarray  # [N, C, 3] f32
    raw_opac: np.ndarray  # [N] f32

    @property
    def n(self) -> int:
        return int(self.transforms.shape[0])

    @property
    def sh_degree(self) -> int:
        c = self.sh.shape[1]
        return int(round(c ** 0.5)) - 1


def rgb_to_sh(rgb: np.ndarray) -> np.ndarray:
    return ((rgb - np.float32(0.5)) / SH_C0).astype(np.float32)


def random_splats(n: int, seed: int, *, mean_lo: float, mean_hi: float, log_scale_mu: float,
                  log_scale_sigma: float, opac_mu: float, opac_sigma: float, sh_degree: int,
                  band_sigma: float = 0.05) -> SplatSet:
    rng = np.random.default_rng(seed)
    t = np.empty((n, 10), dtype=np.float32)
    t[:, 0:3] = rng.uniform(mean_lo, mean_hi, size=(n, 3)).astype(np.float32)
    q = rng.standard_normal((n, 4), dtype=np.float32)
    q /= np.linalg.norm(q, axis=1, keepdims=True)
    t[:, 3:7] = q
    t[:, 7:10] = (log_scale_mu + log_scale_sigma * rng.standard_normal((n, 3), dtype=np.float32))
    raw = (opac_mu + opac_sigma * rng.standard_normal(n, dtype=np.float32)).astype(np.float32)
    c = (sh_degree + 1) ** 2
    sh = np.empty((n, c, 3), dtype=np.float32)
    sh[:, 0, :] = rgb_to_sh(rng.uniform(0.0, 1.0, size=(n, 3)).astype(np.float32))
    if c > 1:
        sh[:, 1:, :] = band_sigma * rng.standard_normal((n, c - 1, 3), dtype=np.float32)
    return SplatSet(t, sh, raw)


def circle_cameras(count: int, radius: float, height: float, width: int, img_h: int,
                   focal: float) -> list[Camera]:
    cams = []
    for i in range(count):
        a = 2.0 * np.pi * i / count
        pos = (radius * np.cos(a), radius * np.sin(a), height)
        cams.append(look_at(pos, (0.0, 0.0, 0.0), width, img_h, focal))
    return cams


def sphere_cameras(count: int, radius: float, width: int, img_h: int, focal: float,
                   seed: int, jitter: float = 0.05) -> list[Camera]:
    """Fibonacci-sphere directions with a seeded radial and angular jitter."""
    rng = np.random.default_rng(seed)
    cams = []
    golden = np.pi * (3.0 - np.sqrt(5.0))
    for i in range(count):
        z = 1.0 - 2.0 * (i + 0.5) / count
        r = np.sqrt(max(0.0, 1.0 - z * z))
        a = golden * i
        d = np.array([r * np.cos(a), r * np.sin(a), z]) + jitter * rng.standard_normal(3)
        d /= np.linalg.norm(d)
        rad = radius * (1.0 + jitter * rng.standard_normal())
        target = 0.1 * rng.standard_normal(3)
        cams.append(look_at(d * rad, target, width, img_h, focal))
    return cams


# --- the benchmark configurations -------------------------------------------------

def config_tiny(seed: int = 1):
    """Config 0: 20k SH-0 splats, 12 views of 256x256 on a circle (r 4, h 0.5)."""
    sp = random_splats(20_000, seed, mean_lo=-1.0, mean_hi=1.0, log_scale_mu=-4.0,
                       log_scale_sigma=0.5, opac_mu=0.0, opac_sigma=1.0, sh_degree=0)
    target = random_splats(20_000, seed + 1000, mean_lo=-1.0, mean_hi=1.0, log_scale_mu=-4.0,
                           log_scale_sigma=0.5, opac_mu=0.0, opac_sigma=1.0, sh_degree=0)
    cams = circle_cameras(12, 4.0, 0.5, 256, 256, 256.0)
    return sp, target, cams


def config_microbench(seed: int = 2, n: int = 1_000_000):
    """Config 1: 1M SH-3 splats in [-3,3]^3, one 1920x1080 view at distance 6."""
    sp = random_splats(n, seed, mean_lo=-3.0, mean_hi=3.0, log_scale_mu=-4.5,
                       log_scale_sigma=0.6, opac_mu=0.0, opac_sigma=1.5, sh_degree=3)
    cam = look_at((6.0, 0.0, 0.0), (0.0, 0.0, 0.0), 1920, 1080, 1600.0)
    return sp, cam


def config_train(seed: int = 3, n: int = 3_000_000, views: int = 200):
    """Config 2: 3M SH-3 splats in [-5,5]^3 (config-1 distributions), 200 views
    of 1600x1060 on a jittered sphere of radius 8, fx = fy = 1300."""
    sp = random_splats(n, seed, mean_lo=-5.0, mean_hi=5.0, log_scale_mu=-4.5,
                       log_scale_sigma=0.6, opac_mu=0.0, opac_sigma=1.5, sh_degree=3)
    cams = sphere_cameras(views, 8.0, 1600, 1060, 1300.0, seed + 17)
    return sp, cams


def config_multiview(seed: int = 4, n: int = 6_000_000, views: int = 8):
    """Config 3: 6M SH-3 splats, a global batch of 8 views at 1920x1080."""
    sp = random_splats(n, seed, mean_lo=-5.0, mean_hi=5.0, log_scale_mu=-4.5,
                       log_scale_sigma=0.6, opac_mu=0.0, opac_sigma=1.5, sh_degree=3)
    cams = sphere_cameras(views, 8.0, 1920, 1080, 1600.0, seed + 17)
    return sp, cams


def config_stress(seed: int = 5, n: int = 10_000_000):
    """Config 4: 10M large splats (log-scale N(-2.5, 0.5), logits N(1, 1)),
    one 3840x2160 view, fx = fy = 3000."""
    sp = random_splats(n, seed, mean_lo=-5.0, mean_hi=5.0, log_scale_mu=-2.5,
                       log_scale_sigma=0.5, opac_mu=1.0, opac_sigma=1.0, sh_degree=3)
    cam = look_at((10.0, 0.0, 0.0), (0.0, 0.0, 0.0), 3840, 2160, 3000.0)
    return sp, cam


def pack_rgba8(img: np.ndarray) -> np.ndarray:
    """[H, W, 3|4] floats in [0, 1] -> packed RGBA8 [H, W] u32 (r in the low
    byte), the reference's ground-truth format
    (crates/splat-train-dataset/src/scene.rs:165-167).  Alpha is 255 when the
    image has 3 channels."""
    h, w = img.shape[:2]
    q = np.clip(np.rint(img[..., :3] * 255.0), 0, 255).astype(np.uint32)
    a = np.full((h, w), 255, dtype=np.uint32) if img.shape[2] == 3 else \
        np.clip(np.rint(img[..., 3] * 255.0), 0, 255).astype(np.uint32)
    return (q[..., 0] | (q[..., 1] << 8) | (q[..., 2] << 16) | (a << 24)).astype(np.uint32)
