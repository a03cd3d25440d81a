"""The Mip-Splatting 3D-filter floor (min_scale) on the GPU against the oracle.

The reference gives every splat a world-space scale floor of sqrt(factor)
pixel sizes at its nearest training camera whenever the training images have
at most 300k pixels (crates/splat-train/src/train.rs:347-387, 2040-2056),
folds it into scales and opacity at render and in the fused update
(src/kernels/helpers.rs:516-553, src/bwd/kernels/project_update.rs), and bakes
it into the parameters before each refine and at export
(gaussian_splats.rs:165-188, 390-402).  Checked here: the floor and the bake
bit for bit, a floored render and the fused 8-bit-moment step bit for bit
given the same rasterizer gradient, whole training steps at configs[0] within
the training tolerance, and the trainer attaching a fresh floor at refine."""
import numpy as np
import pytest
import torch

import oracle
from vauss_b200 import checkpoint, ops, scenes
from vauss_b200.trainer import SceneBatch, Splats, SplatTrainer, TrainConfig
from tests.helpers import assert_bits_equal, medium_scene
from tests.oracle_trainer import OracleTrainer
from tests.test_gpu_parity import _oracle_q8_step, _q8_dev, _q8_host

pytestmark = pytest.mark.gpu


def _np(t):
    return t.detach().cpu().numpy()


def _cam_rows(cams):
    return np.array([[*c.position, np.float32(1.0) / np.float32(max(c.fx, 1e-6))] for c in cams], np.float32)


def test_min_scale_and_fold_bit_exact(cuda):
    sp, cams = medium_scene(seed=51, n=30_000)
    rows = _cam_rows(cams + scenes.circle_cameras(5, 3.0, 0.4, 256, 256, 250.0))
    want = oracle.min_scale(sp.transforms, rows, 0.1)
    got = ops.min_scale(torch.from_numpy(sp.transforms).to(cuda), torch.from_numpy(rows).to(cuda), 0.1)
    assert_bits_equal(_np(got), want, "min_scale")
    assert np.all(want > 0) and np.all(np.isfinite(want))
    # fold it in (and a coarse floor, so that the opacity clamp engages too)
    for scale in (1.0, 50.0):
        ms = (want * np.float32(scale)).astype(np.float32)
        wt, wo = oracle.fold_min_scale(sp.transforms, sp.raw_opac, ms)
        t, o = torch.from_numpy(sp.transforms).to(cuda), torch.from_numpy(sp.raw_opac).to(cuda)
        ops.fold_min_scale(t, o, torch.from_numpy(ms).to(cuda))
        assert_bits_equal(_np(t), wt, f"folded transforms x{scale}")
        assert_bits_equal(_np(o), wo, f"folded opacities x{scale}")
        assert np.all(wt[:, 7:10] >= sp.transforms[:, 7:10])


def test_floor_render_and_q8_step_bit_exact(cuda):
    sp, cams = medium_scene(seed=52, n=20_000)
    cam = cams[0]
    ms = oracle.min_scale(sp.transforms, _cam_rows(cams), 0.1) * np.float32(3.0)
    cfg_o = oracle.make_cfg(3, mip=True, has_min_scale=True)
    ref = oracle.render_forward(cam, cfg_o, sp, min_scale=ms)
    cfg = ops.render_cfg(3, mip=True, has_min_scale=True)
    t, sh, o = (torch.from_numpy(x).to(cuda) for x in (sp.transforms, sp.sh, sp.raw_opac))
    msd = torch.from_numpy(ms).to(cuda)
    out = ops.render(cam, cfg, t, sh, o, min_scale=msd)
    torch.cuda.synchronize()
    assert out.num_visible == ref["proj"]["num_visible"]
    assert_bits_equal(_np(out.frame.field("opacities")), ref["proj"]["opacities"], "floored opacities")
    assert_bits_equal(_np(out.out_img), ref["out_img"], "image")
    # the fused step with the floor, given one rasterizer gradient
    rng = np.random.default_rng(3)
    n, v = sp.n, ref["proj"]["num_visible"]
    vc = (1e-3 * rng.standard_normal((v, 10))).astype(np.float32)
    mom = dict(t=_q8_host(n * 10, rng), sh=_q8_host(sp.sh.size, rng), o=_q8_host(n, rng))
    lr_t = np.float32([1e-3] * 3 + [2e-3] * 4 + [5e-3] * 3)
    # the oracle composite with the floor in its VJP
    grads, refine = oracle.vjp_dense(cam, cfg_o, sp.transforms, sp.sh, sp.raw_opac, ref["proj"]["compact_from_global"],
                                     vc, min_scale=ms)
    grads_plain, _ = oracle.vjp_dense(cam, cfg_o, sp.transforms, sp.sh, sp.raw_opac,
                                      ref["proj"]["compact_from_global"], vc)
    assert not np.array_equal(grads[:, 7:11], grads_plain[:, 7:11])  # the floor changes the scale gradients
    b1, b2, inv1, inv2 = ops.adam_coefficients(4)
    width = grads.shape[1]
    res_t = oracle.adam_q8(sp.transforms, grads, width, 0, 10, mom["t"]["mc"], mom["t"]["vc"], mom["t"]["ms"],
                           mom["t"]["vs"], lr_t, 1.0, b1, b2, inv1, inv2, 1e-15, 4 ^ (10 << 24))
    res_o = oracle.adam_q8(sp.raw_opac, grads, width, width - 1, 1, mom["o"]["mc"], mom["o"]["vc"], mom["o"]["ms"],
                           mom["o"]["vs"], np.float32([5e-2]), 1.0, b1, b2, inv1, inv2, 1e-15, 4 ^ (1 << 24))
    mt, msh, mo = _q8_dev(mom["t"], cuda), _q8_dev(mom["sh"], cuda), _q8_dev(mom["o"], cuda)
    rn = torch.zeros(n, device=cuda)
    ops.step_q8(out.frame, cfg, t, sh, o, torch.from_numpy(vc).to(cuda), mt, msh, mo,
                ops.q8_cfg(4, lr_t, 2.5e-3, 2.5e-4, 5e-2), visible=out.visible, refine_norm=rn, min_scale=msd)
    torch.cuda.synchronize()
    assert_bits_equal(_np(t), res_t[0].reshape(n, 10), "transforms")
    assert_bits_equal(_np(o), res_o[0], "raw opacities")
    assert_bits_equal(_np(mt.m_codes), res_t[1], "transforms m codes")
    assert_bits_equal(_np(rn), refine, "refine weights")


def test_step_q8_wants_the_floor_the_frame_was_rendered_with(cuda):
    sp, cams = medium_scene(seed=53, n=2_000)
    cfg = ops.render_cfg(3, mip=True, has_min_scale=True)
    t, sh, o = (torch.from_numpy(x).to(cuda) for x in (sp.transforms, sp.sh, sp.raw_opac))
    ms = torch.full((sp.n,), 1e-3, device=cuda)
    out = ops.render(cams[0], cfg, t, sh, o, min_scale=ms)
    vc = torch.zeros(max(out.num_visible, 1), 10, device=cuda)
    moms = [ops.Q8Moments(sp.n * 10, cuda), ops.Q8Moments(sp.sh.size, cuda), ops.Q8Moments(sp.n, cuda)]
    with pytest.raises(Exception, match="min_scale"):
        ops.step_q8(out.frame, cfg, t, sh, o, vc, *moms, ops.q8_cfg(1, [1e-3] * 10, 1e-3, 1e-4, 1e-2))


def _targets(tgt, cams):
    cfg = oracle.make_cfg(tgt.sh_degree, mip=True)
    return [scenes.pack_rgba8(np.clip(oracle.render_forward(c, cfg, tgt)["out_img"][..., :3], 0, 1)) for c in cams]


def test_training_with_floor_matches_oracle_tiny_config(cuda):
    """configs[0] (20k SH-0 splats, 12 views of 256x256: below 300k pixels, so
    the reference trains with the floor): three steps with the floor on."""
    sp, tgt, cams = scenes.config_tiny()
    gts = _targets(tgt, cams)
    cfg = TrainConfig(optimizer="q8", total_train_iters=100, lr_mean=1e-3, lr_mean_end=1e-4)
    kw = dict(scene_extent=1.0, median_scale=0.02, seed=9)
    gpu = SplatTrainer(cfg, cuda, **kw)
    gpu.set_view_cams(cams)
    assert gpu.floor_applies(0)
    ora = OracleTrainer(cfg, sp, **kw)
    ms = ops.min_scale(torch.from_numpy(sp.transforms).to(cuda), gpu.view_cams, cfg.min_scale_factor)
    ora.min_scale = oracle.min_scale(sp.transforms, _cam_rows(cams), cfg.min_scale_factor)
    assert_bits_equal(_np(ms), ora.min_scale, "floor")
    base = Splats.from_numpy(sp, cuda)
    splats = Splats(base.transforms, base.sh_coeffs, base.raw_opacities, ms)
    for k in range(3):
        cam = cams[k]
        splats, st = gpu.step(SceneBatch(torch.from_numpy(gts[k].view(np.int32)).to(cuda), cam, k), splats)
        want_loss = ora.step_oracle(gts[k], cam)
        assert abs(float(st.loss.item()) - want_loss) <= 1e-5 * max(1.0, abs(want_loss)), (k, st.loss, want_loss)
    torch.cuda.synchronize()

    def close(got, want, what):
        err = np.abs(got - want)
        bound = 2e-5 + 1e-4 * np.abs(want)
        assert np.mean(err > bound) <= 1e-4, (what, float(np.mean(err > bound)))
    close(_np(splats.transforms), ora.sp.transforms, "transforms")
    close(_np(splats.sh_coeffs), ora.sp.sh, "sh")
    close(_np(splats.raw_opacities), ora.sp.raw_opac, "raw_opacities")


def test_refine_bakes_and_refreshes_the_floor(cuda, tmp_path):
    sp, tgt, cams = scenes.config_tiny()
    gts = [torch.from_numpy(g.view(np.int32)).to(cuda) for g in _targets(tgt, cams)]
    cfg = TrainConfig(optimizer="q8", total_train_iters=100, refine_every=10, lr_mean=1e-3, lr_mean_end=1e-3,
                      background_noise_strength=0.0)
    tr = SplatTrainer(cfg, cuda, scene_extent=1.0, median_scale=0.02)
    tr.set_view_cams(cams)
    splats = Splats.from_numpy(sp, cuda)
    for k in range(1, 26):
        splats, st = tr.step(SceneBatch(gts[k % 12], cams[k % 12], k % 12), splats)
        if tr.should_refine(k):
            before = splats.min_scale
            splats, _ = tr.refine(k, splats)
            assert splats.min_scale is not None and splats.min_scale.shape[0] == splats.num_splats
            fresh = oracle.min_scale(_np(splats.transforms), _cam_rows(cams), cfg.min_scale_factor)
            assert_bits_equal(_np(splats.min_scale), fresh, f"floor after refine {k}")
            if before is not None:
                assert splats.min_scale is not before
    assert np.isfinite(float(st.loss.item()))
    # export bakes the floor; a resumable checkpoint keeps raw values and the floor
    rows = checkpoint.ply_rows(splats)
    t, o = splats.transforms.clone(), splats.raw_opacities.clone()
    ops.fold_min_scale(t, o, splats.min_scale)
    assert np.allclose(rows[:, 3:6], _np(t)[:, 7:10]) and np.allclose(rows[:, 6], _np(o))
    checkpoint.save_checkpoint(str(tmp_path / "ck"), tr, splats)
    tr2, sp2 = checkpoint.load_checkpoint(str(tmp_path / "ck"), cuda)
    assert_bits_equal(_np(sp2.min_scale), _np(splats.min_scale), "reloaded floor")
    assert_bits_equal(_np(sp2.transforms), _np(splats.transforms), "reloaded raw transforms")
    assert_bits_equal(_np(sp2.raw_opacities), _np(splats.raw_opacities), "reloaded raw opacities")
