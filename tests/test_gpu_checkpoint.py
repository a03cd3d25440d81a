"""Checkpoint I/O on the GPU: PLY rows bit-exact against the oracle (f32 and
f16 SH, degenerate quaternions, several chunks, pinned and pageable
destinations), export -> import round trips (the reference's own round-trip
tests, export.rs:543-604, import.rs:722-800), defaults for absent
properties, colour overrides, subsampling, and a resumed training run."""
import ctypes
import os

import numpy as np
import pytest
import torch

import oracle
from vauss_b200 import checkpoint, ops, scenes
from vauss_b200.trainer import SceneBatch, Splats, SplatTrainer, TrainConfig
from tests.test_cpu_checkpoint import reference_test_splats

pytestmark = pytest.mark.gpu


def _same_rows(got, want):
    """Bit-identical, except that any NaN equals any NaN (x86 keeps a NaN's
    payload through a division, the GPU returns its canonical NaN)."""
    assert got.shape == want.shape
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got.view(np.uint32)[~nan], want.view(np.uint32)[~nan])


def _random_splats(n, degree, seed, half=False):
    rng = np.random.default_rng(seed)
    t = rng.standard_normal((n, 10)).astype(np.float32)
    t[::7, 3:7] = 0.0
    t[::11, 4] = np.nan
    t[::13, 3:7] *= np.float32(1e-30)
    sh = rng.standard_normal((n, (degree + 1) ** 2, 3)).astype(np.float32)
    if half:
        sh = sh.astype(np.float16).astype(np.float32)
    o = rng.standard_normal(n).astype(np.float32)
    return t, sh, o


@pytest.mark.parametrize("degree", [0, 1, 2, 3])
@pytest.mark.parametrize("half", [False, True])
def test_rows_bit_exact(cuda, degree, half):
    t, sh, o = _random_splats(3001, degree, degree + 10 * half, half)
    s = Splats(torch.from_numpy(t).to(cuda), torch.from_numpy(sh).to(cuda).to(torch.float16 if half else torch.float32),
               torch.from_numpy(o).to(cuda))
    _same_rows(checkpoint.ply_rows(s), oracle.ply_encode(t, sh, o))


def test_rows_many_chunks_pinned_and_pageable(cuda):
    n = 600_000  # 248-byte rows: three 64 MB chunks
    t, sh, o = _random_splats(n, 3, 5)
    s = Splats(*(torch.from_numpy(a).to(cuda) for a in (t, sh, o)))
    want = oracle.ply_encode(t, sh, o)
    _same_rows(checkpoint.ply_rows(s), want)
    pinned = torch.empty(want.nbytes, dtype=torch.uint8).pin_memory()
    ctx = ops.context(cuda)
    ctx.check(ctx.lib.vs_ply_encode(ctx.h, n, 3, ops._ptr(s.transforms), ops._ptr(s.sh_coeffs), 0,
                                    ops._ptr(s.raw_opacities), ctypes.c_void_p(pinned.data_ptr())))
    _same_rows(pinned.numpy().view(np.float32).reshape(want.shape), want)


@pytest.mark.parametrize("degree", [0, 1, 2, 3])
def test_round_trip(cuda, degree, tmp_path):
    t, sh, o = reference_test_splats(degree, 100)
    s = Splats(*(torch.from_numpy(a).to(cuda) for a in (t, sh, o)))
    path = os.path.join(tmp_path, "s.ply")
    checkpoint.write_ply(path, s, up_axis=(0.0, 0.0, 1.0))
    back, meta = checkpoint.load_ply(path, cuda)
    assert back.num_splats == 100 and back.sh_degree == degree
    assert meta.up_axis == (0.0, 0.0, 1.0) and meta.render_mode == "default" and meta.total_splats == 100
    np.testing.assert_array_equal(back.sh_coeffs.cpu().numpy(), sh)
    np.testing.assert_array_equal(back.transforms.cpu().numpy(), t)  # unit quaternions: exact
    np.testing.assert_array_equal(back.raw_opacities.cpu().numpy(), o)
    # bytes in, same bytes out
    assert checkpoint.splat_to_ply(back, up_axis=(0.0, 0.0, 1.0)) == open(path, "rb").read()


def test_import_subsample_defaults_and_colours(cuda):
    rng = np.random.default_rng(2)
    n = 10
    # x y z as double, colours as uchar, no rotation / scale / opacity / SH
    dt = np.dtype([("x", "<f8"), ("y", "<f8"), ("z", "<f8"), ("red", "u1"), ("green", "u1"), ("blue", "u1")])
    rows = np.zeros(n, dt)
    for a in ("x", "y", "z"):
        rows[a] = rng.standard_normal(n)
    for a in ("red", "green", "blue"):
        rows[a] = rng.integers(0, 256, n)
    head = ("ply\nformat binary_little_endian 1.0\ncomment Vertical axis: x\nelement vertex 10\n"
            "property double x\nproperty double y\nproperty double z\nproperty uchar red\n"
            "property uchar green\nproperty uchar blue\nend_header\n").encode()
    s, meta = checkpoint.load_ply(head + rows.tobytes(), cuda)
    assert meta.up_axis == (1.0, 0.0, 0.0) and s.sh_degree == 0
    t = s.transforms.cpu().numpy()
    np.testing.assert_array_equal(t[:, 0], rows["x"].astype(np.float32))
    np.testing.assert_array_equal(t[:, 3:7], np.tile(np.float32([1, 0, 0, 0]), (n, 1)))
    np.testing.assert_array_equal(t[:, 7:], np.full((n, 3), -4.0, np.float32))
    np.testing.assert_array_equal(s.raw_opacities.cpu().numpy(), np.zeros(n, np.float32))
    want_dc = (rows["red"].astype(np.float32) / np.float32(254) - np.float32(0.5)) / np.float32(checkpoint.SH_C0)
    np.testing.assert_array_equal(s.sh_coeffs.cpu().numpy()[:, 0, 0], want_dc)
    # only positions: SH 0.5; every third row with subsample 3
    pos = np.zeros(n, [("x", "<f4"), ("y", "<f4"), ("z", "<f4")])
    pos["x"] = np.arange(n)
    head2 = ("ply\nformat binary_little_endian 1.0\nelement vertex 10\nproperty float x\nproperty float y\n"
             "property float z\nend_header\n").encode()
    s2, meta2 = checkpoint.load_ply(head2 + pos.tobytes(), cuda, subsample_points=3)
    assert s2.num_splats == 3 and meta2.total_splats == 3
    np.testing.assert_array_equal(s2.transforms.cpu().numpy()[:, 0], np.float32([2, 5, 8]))
    np.testing.assert_array_equal(s2.sh_coeffs.cpu().numpy(), np.full((3, 1, 3), 0.5, np.float32))
    with pytest.raises(NotImplementedError):
        checkpoint.load_ply(head2.replace(b"binary_little_endian", b"ascii") + pos.tobytes(), cuda)


def test_resumed_training_matches(cuda, tmp_path):
    """Six steps, checkpoint, six more; a trainer loaded from the checkpoint
    takes the same six steps to the same parameters (within the training
    tolerance: the backward sums with float atomics)."""
    sp, tgt, cams = scenes.config_tiny()
    cfg_o = oracle.make_cfg(0, mip=True)
    gts = [torch.from_numpy(scenes.pack_rgba8(np.clip(oracle.render_forward(c, cfg_o, tgt)["out_img"][..., :3], 0, 1))
                            .view(np.int32)).to(cuda) for c in cams]
    cfg = TrainConfig(optimizer="q8", total_train_iters=100, background_noise_strength=0.02)
    tr = SplatTrainer(cfg, cuda, scene_extent=1.0, median_scale=0.02)
    splats = Splats.from_numpy(sp, cuda)
    for k in range(6):
        splats, _ = tr.step(SceneBatch(gts[k % 12], cams[k % 12], k % 12), splats)
    d = os.path.join(tmp_path, "ck")
    checkpoint.save_checkpoint(d, tr, splats)
    tr2, splats2 = checkpoint.load_checkpoint(d, cuda)
    torch.cuda.synchronize()
    assert torch.equal(splats2.transforms, splats.transforms) and torch.equal(splats2.sh_coeffs, splats.sh_coeffs)
    for key in ("t", "sh", "o"):
        assert torch.equal(tr2.optim[key].m_codes, tr.optim[key].m_codes)
        assert torch.equal(tr2.optim[key].v_scales, tr.optim[key].v_scales)
    assert tr2.step_count == tr.step_count and tr2.optim["time"] == tr.optim["time"]
    for k in range(6, 12):
        b = SceneBatch(gts[k % 12], cams[k % 12], k % 12)
        splats, st1 = tr.step(b, splats)
        splats2, st2 = tr2.step(b, splats2)
        assert abs(float(st1.loss.item()) - float(st2.loss.item())) <= 1e-5
    a, b = splats.transforms.cpu().numpy(), splats2.transforms.cpu().numpy()
    err = np.abs(a - b)
    assert np.mean(err > 2e-5 + 1e-4 * np.abs(a)) <= 1e-3 and float(err.max()) < 1e-2
