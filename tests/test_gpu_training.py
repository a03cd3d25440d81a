"""Whole training steps on the GPU (SplatTrainer.step, the public API) against
the oracle's restatement of the same steps, in both optimizer modes, plus
render invariants and argument validation through the C ABI."""
import math

import numpy as np
import pytest
import torch

import oracle
from vauss_b200 import _native, ops, scenes
from vauss_b200.camera import Camera
from vauss_b200.trainer import SceneBatch, Splats, SplatTrainer, TrainConfig
from tests.helpers import assert_bits_equal, medium_scene
from tests.oracle_trainer import OracleTrainer

pytestmark = pytest.mark.gpu


def _targets(tgt, cams):
    cfg = oracle.make_cfg(tgt.sh_degree, mip=True)
    return [scenes.pack_rgba8(np.clip(oracle.render_forward(c, cfg, tgt)["out_img"][..., :3], 0, 1)) for c in cams]


@pytest.mark.parametrize("mode", ["q8", "reference"])
def test_training_steps_match_oracle(cuda, mode):
    sp, cams = medium_scene(seed=31, n=20_000, sh_degree=3)
    tgt, _ = medium_scene(seed=32, n=20_000, sh_degree=3)
    gts = _targets(tgt, cams)
    cfg = TrainConfig(optimizer=mode, total_train_iters=100, lr_mean=1e-3, lr_mean_end=1e-4)
    kw = dict(scene_extent=1.0, median_scale=0.02, seed=5)
    gpu = SplatTrainer(cfg, cuda, **kw)
    ora = OracleTrainer(cfg, sp, **kw)
    splats = Splats.from_numpy(sp, cuda)
    for k in range(3):
        cam = cams[k % 2]
        splats, st = gpu.step(SceneBatch(torch.from_numpy(gts[k % 2].view(np.int32)).to(cuda), cam), splats)
        want_loss = ora.step_oracle(gts[k % 2], cam)
        assert abs(float(st.loss.item()) - want_loss) <= 1e-5 * max(1.0, abs(want_loss)), (k, st.loss, want_loss)
    torch.cuda.synchronize()
    # The backward's atomics sum in another order, so a stochastic-rounding
    # decision of a moment code can flip (about one value in 1e5); such a flip
    # moves a parameter by at most ~lr * 8/127.  Everything else agrees to
    # 2e-5.
    def close(got, want, what):
        err = np.abs(got - want)
        bound = 2e-5 + 1e-4 * np.abs(want)
        assert np.mean(err > bound) <= 1e-4, (what, float(np.mean(err > bound)))
        assert float(err.max()) <= 2e-4 + 1e-3 * float(np.abs(want).max()), (what, float(err.max()))
    close(splats.transforms.cpu().numpy(), ora.sp.transforms, "transforms")
    close(splats.sh_coeffs.float().cpu().numpy(), ora.sh_values(), "sh")
    close(splats.raw_opacities.cpu().numpy(), ora.sp.raw_opac, "raw_opacities")
    np.testing.assert_allclose(gpu.record.vis_count.cpu().numpy(), ora.vis)


def test_training_reduces_loss_tiny_config(cuda):
    """Config 0 (20k SH-0 splats, 12 views of 256x256) trains: the loss falls."""
    sp, tgt, cams = scenes.config_tiny()
    gts = [torch.from_numpy(g.view(np.int32)).to(cuda) for g in _targets(tgt, cams)]
    cfg = TrainConfig(optimizer="q8", total_train_iters=100, lr_mean=1e-3, lr_mean_end=1e-3, lr_scale=5e-3,
                      lr_opac=5e-2, lr_coeffs_dc=2.5e-3, background_noise_strength=0.0)
    tr = SplatTrainer(cfg, cuda, scene_extent=1.0, median_scale=0.02)
    splats = Splats.from_numpy(sp, cuda)
    losses = []
    for k in range(100):
        splats, st = tr.step(SceneBatch(gts[k % 12], cams[k % 12], k % 12), splats)
        losses.append(float(st.loss.item()))
    first, last = np.mean(losses[:12]), np.mean(losses[-12:])
    assert last < first, (first, last)
    assert all(math.isfinite(x) for x in losses)
    assert bool(torch.isfinite(splats.transforms).all())


def _cam_z(w, h, fov=0.5, z=-5.0):
    f = (w / 2.0) / math.tan(fov / 2.0)
    return Camera(R=np.eye(3, dtype=np.float32), t=np.float32([0.0, 0.0, -z]), fx=f, fy=f, cx=w / 2.0, cy=h / 2.0,
                  width=w, height=h)


def _render_gpu(sp, cam, dev, bg=(0.0, 0.0, 0.0)):
    s = Splats.from_numpy(sp, dev)
    out = ops.render(cam, ops.render_cfg(sp.sh_degree, mip=False, background=bg), s.transforms, s.sh_coeffs,
                     s.raw_opacities)
    torch.cuda.synchronize()
    return out


def test_gpu_render_invariants(cuda):
    from tests.test_cpu_oracle import _cat, _rng_scene
    cam = _cam_z(256, 256)
    vis = _rng_scene(5_000, 1.5, (-3.5, -1.5), (0.0, 3.0), 0xBEEF)
    hidden = _rng_scene(20_000, 1.0, (-1.0, 1.0), (-20.0, -20.0), 0xDEAD)
    for i in range(hidden.n):
        if i % 3 == 1:
            hidden.transforms[i, :3] = (0.0, 0.0, -1000.0)
        elif i % 3 == 2:
            hidden.transforms[i, :3] = (1e6, 1e6, 10.0)
            hidden.raw_opac[i] = 3.0
    base = _render_gpu(vis, cam, cuda).out_img.cpu().numpy()
    again = _render_gpu(vis, cam, cuda).out_img.cpu().numpy()
    assert_bits_equal(again, base, "determinism")
    assert_bits_equal(_render_gpu(_cat(vis, hidden), cam, cuda).out_img.cpu().numpy(), base, "hidden suffix")
    assert_bits_equal(_render_gpu(_cat(hidden, vis), cam, cuda).out_img.cpu().numpy(), base, "culled prefix")
    bad = scenes.SplatSet(vis.transforms.copy(), vis.sh.copy(), vis.raw_opac.copy())
    bad.transforms[:, 3:7] = 0.0
    bad.transforms[::5, 1] = np.nan
    assert_bits_equal(_render_gpu(_cat(vis, bad), cam, cuda).out_img.cpu().numpy(), base, "zero quats / NaN means")


def test_gpu_many_large_splats_no_dropped_tiles(cuda):
    from tests.test_cpu_oracle import _rng_scene
    cam = _cam_z(128, 128)
    sp = _rng_scene(200_000, 0.5, (-1.0, 2.5), (-2.0, 2.0), 17)
    out = _render_gpu(sp, cam, cuda)
    img = out.out_img.cpu().numpy()
    assert np.isfinite(img).all()
    alpha = img[..., 3].reshape(8, 16, 8, 16).sum(axis=(1, 3))
    assert (alpha >= 1e-4).all()
    assert out.num_intersections > 1_000_000


def test_gpu_zero_and_single_splat(cuda):
    cam = _cam_z(40, 24, z=-3.0)
    empty = scenes.SplatSet(np.zeros((0, 10), np.float32), np.zeros((0, 1, 3), np.float32), np.zeros(0, np.float32))
    t = torch.zeros(0, 10, device=cuda)
    out = ops.render(cam, ops.render_cfg(0, mip=False, background=(0.7, 0.3, 0.1)), t,
                     torch.zeros(0, 1, 3, device=cuda), torch.zeros(0, device=cuda))
    img = out.out_img.cpu().numpy()
    assert np.allclose(img[..., :3], np.float32([0.7, 0.3, 0.1])) and np.all(img[..., 3] == 0)
    assert out.num_visible == 0 and out.num_intersections == 0
    del empty
    one = scenes.SplatSet(np.float32([[0, 0, 0, 1, 0, 0, 0, -1.5, -1.5, -1.5]]), np.ones((1, 1, 3), np.float32),
                          np.float32([2.0]))
    ref = oracle.render_forward(cam, oracle.make_cfg(0, mip=False), one)
    got = _render_gpu(one, cam, cuda)
    assert_bits_equal(got.out_img.cpu().numpy(), ref["out_img"], "single splat")


def test_abi_rejects_bad_arguments(cuda):
    sp, cams = medium_scene(n=100, sh_degree=3)
    s = Splats.from_numpy(sp, cuda)
    zero = Camera(R=np.eye(3, dtype=np.float32), t=np.zeros(3, np.float32), fx=1, fy=1, cx=0, cy=0, width=0, height=0)
    with pytest.raises(_native.VsError) as e:
        ops.render(zero, ops.render_cfg(3), s.transforms, s.sh_coeffs, s.raw_opacities,
                   out_img=torch.empty(1, 1, 4, device=cuda))
    assert e.value.status == 1 and "zero image size" in str(e.value)
    ctx = ops.context(cuda)
    fr = ops.Frame(ctx)
    st = ctx.lib.vs_rasterize_backward(ctx.h, fr.h, None, None, None)
    assert st == 1 and b"not been rendered" in ctx.lib.vs_ctx_last_error(ctx.h)
    cfg4 = ops.render_cfg(3)
    cfg4.sh_degree = 4
    cam = cams[0].to_c()
    import ctypes
    st = ctx.lib.vs_render_project(ctx.h, fr.h, ctypes.byref(cam), ctypes.byref(cfg4), 1, None, None, None, None,
                                   None)
    assert st == 5


def test_render_rejects_misaligned_transforms(cuda):
    """Projection reads each 40-byte transforms row in 8-byte pieces; a
    transforms array that starts off an 8-byte boundary is refused before any
    launch."""
    sp, cams = medium_scene(n=300, sh_degree=3)
    s = Splats.from_numpy(sp, cuda)
    t = torch.zeros(300 * 10 + 1, device=cuda)[1:].view(300, 10)  # 4 bytes past an aligned start
    t.copy_(s.transforms)
    with pytest.raises(_native.VsError) as e:
        ops.render(cams[0], ops.render_cfg(3), t, s.sh_coeffs, s.raw_opacities)
    assert e.value.status == 1 and "8-byte aligned" in str(e.value)


def test_render_with_misaligned_sh_matches_aligned(cuda):
    """SH coefficients are read as 16-byte vectors only from an array on a
    16-byte boundary; one 4 bytes off renders through scalar loads, bit for bit
    the same image."""
    sp, cams = medium_scene(n=3000, sh_degree=3)
    s = Splats.from_numpy(sp, cuda)
    sh_off = torch.zeros(3000 * 48 + 1, device=cuda)[1:].view(3000, 16, 3)
    sh_off.copy_(s.sh_coeffs)
    cfg = ops.render_cfg(3, mip=True)
    want = ops.render(cams[0], cfg, s.transforms, s.sh_coeffs, s.raw_opacities).out_img.clone()
    got = ops.render(cams[0], cfg, s.transforms, sh_off, s.raw_opacities).out_img
    torch.cuda.synchronize()
    assert_bits_equal(got.cpu().numpy(), want.cpu().numpy(), "image from a misaligned SH array")


def test_q8_rejects_unaligned_arrays(cuda):
    """The Q8 kernels move parameters and codes in 16-byte pieces; a parameter
    array that starts off a 16-byte boundary is refused before any launch."""
    n = 300
    t = torch.zeros(n * 10 + 1, device=cuda)[1:].view(n, 10)  # 4 bytes past an aligned start
    sh = torch.zeros(n, 16, 3, device=cuda)
    o = torch.zeros(n, device=cuda)
    grads = torch.zeros(n, 10 + 48 + 1, device=cuda)
    mom = [ops.Q8Moments(c, cuda) for c in (n * 10, n * 48, n)]
    q8 = ops.q8_cfg(1, [1e-3] * 10, 1e-3, 1e-4, 1e-2)
    with pytest.raises(_native.VsError) as e:
        ops.adam_q8_dense(3, t, sh, o, grads, *mom, q8)
    assert e.value.status == 1 and "16-byte aligned" in str(e.value)
