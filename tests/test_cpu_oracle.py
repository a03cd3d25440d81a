"""Pins the CPU oracle against the reference's own known-answer tests and
invariants (restated; the reference itself cannot be built or run here).

 * shared exp/log: accuracy against double-precision libm;
 * f16 conversion: exact against numpy's IEEE binary16 rounding;
 * SSIM: against an independent float64 restatement of the reference's test
   reference (crates/splat-train-loss/tests/ssim_reference.rs:26-285): 11x11
   window, sigma 1.5, zero padding, C1 = 0.01^2, C2 = 0.03^2, forward map and
   central finite differences of the mean at probe pixels;
 * loss invariants (crates/splat-train-loss/tests/reference.rs:70-303);
 * render invariants (crates/splat-train-render/src/tests/mod.rs:20-805):
   splats at the camera origin render nothing, determinism, hidden/culled
   splats do not perturb the image, zero quaternions are culled, zero splats
   render the background, no dropped tiles under large splats.
"""
import math

import numpy as np
import pytest

import oracle
from vauss_b200 import scenes
from vauss_b200.camera import Camera

# ---------------------------------------------------------------- math ----


def test_expf_accuracy_and_specials():
    x = np.linspace(-87.0, 88.72, 1_000_001, dtype=np.float32)
    y = oracle.expf(x).astype(np.float64)
    ref = np.exp(x.astype(np.float64))
    rel = np.abs(y - ref) / ref
    assert rel.max() < 2.5e-7  # ~2 ulp
    sp = oracle.expf(np.float32([0.0, -0.0, 88.8, -88.0, np.inf, -np.inf, np.nan]))
    assert sp[0] == 1.0 and sp[1] == 1.0 and np.isinf(sp[2]) and sp[3] == 0.0 and np.isinf(sp[4])
    assert sp[5] == 0.0 and np.isnan(sp[6])


def test_logf_accuracy_and_specials():
    x = np.exp(np.linspace(-100.0, 88.0, 1_000_001)).astype(np.float32)
    y = oracle.logf(x).astype(np.float64)
    ref = np.log(x.astype(np.float64))
    err = np.abs(y - ref)
    assert np.all(err <= 2.5e-7 * np.maximum(np.abs(ref), 1.0))
    near1 = np.float32(1.0) + np.arange(-2000, 2000, dtype=np.float32) * np.float32(2 ** -23)
    e1 = np.abs(oracle.logf(near1).astype(np.float64) - np.log(near1.astype(np.float64)))
    assert np.all(e1 <= 2e-7 * np.abs(np.log(near1.astype(np.float64))) + 1e-12)
    sp = oracle.logf(np.float32([1.0, 0.0, -1.0, np.inf, np.nan, 1e-45]))
    assert sp[0] == 0.0 and sp[1] == -np.inf and np.isnan(sp[2]) and sp[3] == np.inf and np.isnan(sp[4])
    assert abs(sp[5] - math.log(1.401298464324817e-45)) < 1e-4


def test_f16_conversion_matches_ieee():
    rng = np.random.default_rng(0)
    x = np.concatenate([
        rng.standard_normal(200_000).astype(np.float32) * np.float32(10.0) ** rng.integers(-9, 6, 200_000).astype(np.float32),
        np.float32([0.0, -0.0, 65504.0, 65519.0, 65520.0, 1e9, -1e9, 6.1035156e-05, 5.96e-8, 2.98e-8, 2.99e-8,
                    np.inf, -np.inf]),
    ]).astype(np.float32)
    h, back = oracle.f16_roundtrip(x)
    want = x.astype(np.float16)
    assert np.array_equal(h, want.view(np.uint16))
    assert np.array_equal(back, want.astype(np.float32))

# ---------------------------------------------------------------- SSIM ----


def _taps():
    w = np.array([math.exp(-((i - 5.0) ** 2) / (2.0 * 1.5 * 1.5)) for i in range(11)])
    return w / w.sum()


def scene_image(h: int, w: int, seed: int) -> np.ndarray:
    """Deterministic image-like content in [0, 1] (the reference test's
    ``scene``: smooth shading plus hashed texture)."""
    y, x, c = np.meshgrid(np.arange(h, dtype=np.uint64), np.arange(w, dtype=np.uint64),
                          np.arange(3, dtype=np.uint64), indexing="ij")
    m = np.uint64(0xffffffff)
    k = ((y * np.uint64(73_856_093)) & m) ^ ((x * np.uint64(19_349_663)) & m) ^ (
        ((c + np.uint64(seed)) * np.uint64(83_492_791)) & m)
    k ^= k >> np.uint64(13)
    k = (k * np.uint64(0x5bd1_e995)) & m
    k ^= k >> np.uint64(15)
    noise = (k % np.uint64(1000)).astype(np.float64) / 1000.0 - 0.5
    xf, yf, cf = x.astype(np.float64), y.astype(np.float64), c.astype(np.float64)
    v = 0.5 + 0.3 * (np.sin(xf / 7.0 + cf) * np.cos(yf / 5.0)) + 0.15 * noise
    return np.clip(v, 0.0, 1.0)


def _blur(img):
    g = _taps()
    h, w = img.shape[:2]
    pad = np.pad(img, ((0, 0), (5, 5), (0, 0)))
    tmp = sum(g[k] * pad[:, k:k + w] for k in range(11))
    pad = np.pad(tmp, ((5, 5), (0, 0), (0, 0)))
    return sum(g[k] * pad[k:k + h] for k in range(11))


def ssim_map_f64(x, y):
    c1, c2 = 0.01 ** 2, 0.03 ** 2
    mu1, mu2 = _blur(x), _blur(y)
    s1 = _blur(x * x) - mu1 * mu1
    s2 = _blur(y * y) - mu2 * mu2
    s12 = _blur(x * y) - mu1 * mu2
    return ((2 * mu1 * mu2 + c1) * (2 * s12 + c2)) / ((mu1 ** 2 + mu2 ** 2 + c1) * (s1 + s2 + c2))


def _ssim_sum_fd(x, y, r, col, c, eps=1e-5):
    """d sum(SSIM)/d x[r, col, c] by central differences over the affected window."""
    h, w = x.shape[:2]
    rr0, rr1 = max(0, r - 5), min(h, r + 6)
    cc0, cc1 = max(0, col - 5), min(w, col + 6)
    xp, xm = x.copy(), x.copy()
    xp[r, col, c] += eps
    xm[r, col, c] -= eps
    sp = ssim_map_f64(xp, y)[rr0:rr1, cc0:cc1, c].sum()
    sm = ssim_map_f64(xm, y)[rr0:rr1, cc0:cc1, c].sum()
    return (sp - sm) / (2 * eps)


@pytest.mark.parametrize("h,w", [(45, 61), (120, 100)])
def test_ssim_matches_f64_reference(h, w):
    gt = np.round(scene_image(h, w, 3) * 255.0) / 255.0
    tex = scene_image(h, w, 11)
    shifted = gt[:, np.minimum(np.arange(w) + 1, w - 1), :]
    pred = (0.7 * shifted + 0.3 * tex).astype(np.float32)
    pred4 = np.concatenate([pred, np.ones((h, w, 1), np.float32)], axis=2)
    gt_packed = scenes.pack_rgba8(gt)
    lo = oracle.loss_fwd(pred4, gt_packed, 0.0, 1.0, want_map=True)
    ref = ssim_map_f64(pred.astype(np.float64), gt)
    assert np.abs(lo["ssim_map"] - ref).max() < 1e-3
    assert abs(lo["loss"] - ref.mean()) < 1e-4
    dl = oracle.loss_bwd(pred4, gt_packed, lo["coeffs"], 0.0, 1.0)
    n = h * w * 3
    probes = [(0, 0, 0), (0, w - 1, 1), (h - 1, 0, 2), (h - 1, w - 1, 0), (0, w // 2, 1), (h // 2, 0, 2),
              (2, 3, 0), (7, 8, 1), (15, 16, 2), (16, 15, 0), (h // 2, w // 2, 1), (h - 3, w - 6, 2)]
    for (r, col, c) in probes:
        num = _ssim_sum_fd(pred.astype(np.float64), gt, r, col, c)
        ana = float(dl[r, col, c]) * n
        assert abs(num - ana) <= 2e-3 + 0.01 * max(abs(num), abs(ana)), (r, col, c, num, ana)
    assert np.all(dl[..., 3] == 0.0)


def test_ssim_identical_is_one_and_in_range():
    h, w = 40, 56
    rng = np.random.default_rng(1)
    img = rng.integers(0, 256, size=(h, w, 3)).astype(np.float32) / 255.0
    img4 = np.concatenate([img, np.ones((h, w, 1), np.float32)], axis=2)
    packed = scenes.pack_rgba8(img)
    lo = oracle.loss_fwd(img4, packed, 0.0, 1.0, want_map=True)
    assert abs(lo["ssim_map"].mean() - 1.0) < 1e-4
    other = scenes.pack_rgba8(rng.integers(0, 256, size=(h, w, 3)).astype(np.float32) / 255.0)
    lo2 = oracle.loss_fwd(img4, other, 0.0, 1.0, want_map=True)
    assert lo2["ssim_map"].min() >= -1.0 and lo2["ssim_map"].max() <= 1.0
    dl = oracle.loss_bwd(img4, other, lo2["coeffs"], 0.8, -0.2)
    assert np.isfinite(dl).all() and np.abs(dl).max() > 0.0


def test_l1_dssim_weights():
    from vauss_b200.trainer import TrainConfig
    cfg = TrainConfig()
    assert (cfg.l1_weight, cfg.ssim_loss_weight) == (pytest.approx(0.8), pytest.approx(-0.2))

# ------------------------------------------------------------- render ----


def _cam_z(w, h, fov=0.5, z=-5.0):
    f = (w / 2.0) / math.tan(fov / 2.0)
    return Camera(R=np.eye(3, dtype=np.float32), t=np.float32([0.0, 0.0, -z]), fx=f, fy=f, cx=w / 2.0, cy=h / 2.0,
                  width=w, height=h)


def _rng_scene(n, spread, log_scale, opac, seed):
    rng = np.random.default_rng(seed)
    t = np.zeros((n, 10), np.float32)
    t[:, :3] = rng.uniform(-spread, spread, size=(n, 3))
    q = rng.standard_normal((n, 4)).astype(np.float32)
    t[:, 3:7] = q / np.linalg.norm(q, axis=1, keepdims=True)
    t[:, 7:] = rng.uniform(log_scale[0], log_scale[1], size=(n, 3))
    sh = rng.uniform(0, 1, size=(n, 1, 3)).astype(np.float32)
    o = rng.uniform(opac[0], opac[1], size=n).astype(np.float32)
    return scenes.SplatSet(t, sh, o)


def _cat(a, b):
    return scenes.SplatSet(np.concatenate([a.transforms, b.transforms]), np.concatenate([a.sh, b.sh]),
                           np.concatenate([a.raw_opac, b.raw_opac]))


def _render(sp, cam, bg=(0.0, 0.0, 0.0)):
    return oracle.render_forward(cam, oracle.make_cfg(sp.sh_degree, mip=False, bg=bg), sp, bg=bg)


def test_splats_at_camera_render_nothing():
    t = np.zeros((8, 10), np.float32)
    t[:, 3] = 1.0
    t[:, 7:] = 2.0
    cam = Camera(R=np.eye(3, dtype=np.float32), t=np.zeros(3, np.float32), fx=63.0, fy=63.0, cx=16, cy=16,
                 width=32, height=32)
    r = _render(scenes.SplatSet(t, np.ones((8, 1, 3), np.float32), np.zeros(8, np.float32)), cam)
    assert r["proj"]["num_visible"] == 0
    assert np.abs(r["out_img"]).max() == 0.0


def test_render_is_deterministic():
    cam = _cam_z(128, 128)
    sp = _rng_scene(3_000, 2.0, (-3.0, -1.0), (-1.0, 2.0), 0xA11CE)
    a, b = _render(sp, cam), _render(sp, cam)
    assert np.array_equal(a["out_img"], b["out_img"])
    assert np.array_equal(a["binning"]["isect_compact"], b["binning"]["isect_compact"])


def test_hidden_and_culled_splats_do_not_perturb():
    cam = _cam_z(128, 128)
    vis = _rng_scene(2_000, 1.5, (-3.5, -1.5), (0.0, 3.0), 0xBEEF)
    hidden = _rng_scene(3_000, 1.0, (-1.0, 1.0), (-20.0, -20.0), 0xDEAD)
    for i in range(hidden.n):
        if i % 3 == 1:
            hidden.transforms[i, :3] = (0.0, 0.0, -1000.0)  # behind the camera
        elif i % 3 == 2:
            hidden.transforms[i, :3] = (1e6, 1e6, 10.0)  # far off-screen
            hidden.raw_opac[i] = 3.0
    base = _render(vis, cam)["out_img"]
    assert np.array_equal(_render(_cat(vis, hidden), cam)["out_img"], base)
    assert np.array_equal(_render(_cat(hidden, vis), cam)["out_img"], base)  # culled prefix


def test_zero_quaternions_and_nan_positions_are_culled():
    cam = _cam_z(64, 64, z=-3.0)
    valid = _rng_scene(500, 1.0, (-3.0, -1.0), (0.0, 2.0), 0xDEAD)
    bad = scenes.SplatSet(valid.transforms.copy(), valid.sh.copy(), valid.raw_opac.copy())
    bad.transforms[:, 3:7] = 0.0
    bad.transforms[::7, 0] = np.nan
    base = _render(valid, cam)["out_img"]
    r = _render(_cat(valid, bad), cam)
    assert np.array_equal(r["out_img"], base)
    assert r["proj"]["num_visible"] == _render(valid, cam)["proj"]["num_visible"]


def test_zero_splats_render_background():
    cam = _cam_z(32, 32, z=-3.0)
    empty = scenes.SplatSet(np.zeros((0, 10), np.float32), np.zeros((0, 1, 3), np.float32), np.zeros(0, np.float32))
    r = _render(empty, cam, bg=(0.7, 0.3, 0.1))
    assert np.allclose(r["out_img"][..., :3], np.float32([0.7, 0.3, 0.1]), atol=1e-6)
    assert np.all(r["out_img"][..., 3] == 0.0)


def test_no_dropped_tiles_under_large_splats():
    cam = _cam_z(64, 64)
    sp = _rng_scene(3_000, 0.5, (-1.0, 1.0), (-2.0, 2.0), 3)
    img = _render(sp, cam)["out_img"]
    assert np.isfinite(img).all()
    alpha = img[..., 3].reshape(4, 16, 4, 16).sum(axis=(1, 3))
    assert (alpha >= 1e-4).all()
