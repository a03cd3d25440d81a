"""Refinement on the GPU: the decision table, the split (with filler rows),
the opacity decay and the moment row resets against the oracle bit for bit,
and training that refines in the middle (counts, shapes, finite losses)."""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from vauss_b200 import _native as N
from vauss_b200 import ops, scenes
from vauss_b200.refine import MIN_OPACITY
from vauss_b200.trainer import SceneBatch, Splats, SplatTrainer, TrainConfig
from tests.helpers import assert_bits_equal

pytestmark = pytest.mark.gpu


def _scene(n, seed):
    rng = np.random.default_rng(seed)
    t = rng.standard_normal((n, 10)).astype(np.float32)
    t[:, 7:10] = rng.normal(-4.0, 1.0, (n, 3)).astype(np.float32)
    t[::97, 0] = 5e3          # far outside the bounds
    t[::89, 8] = 12.0         # enormous scale
    t[::83, 4] = np.nan       # non-finite
    sh = (0.3 * rng.standard_normal((n, 16, 3))).astype(np.float32)
    sh[::79, 3, 1] = np.inf
    o = rng.normal(0.0, 3.0, n).astype(np.float32)
    return t, sh, o, rng


def _d(x, dev):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


def test_refine_table_bit_exact(cuda):
    n = 5000
    t, sh, o, rng = _scene(n, 1)
    w = rng.random(n).astype(np.float32)
    vis = (rng.random(n) < 0.7).astype(np.float32) * rng.integers(1, 4, n).astype(np.float32)
    scr = (rng.random(n) * 0.8).astype(np.float32)
    want = oracle.refine_table(t, sh, o, w, vis, scr, MIN_OPACITY, 50.0, [0.1, -0.2, 0.3], 0.5)
    ctx = ops.context(cuda)
    cfg = N.RefineCfg()
    cfg.min_opacity, cfg.max_bound, cfg.split_at_screen_size = MIN_OPACITY, 50.0, 0.5
    cfg.center[0], cfg.center[1], cfg.center[2] = 0.1, -0.2, 0.3
    table = torch.empty(n, 8, device=cuda)
    # every device array stays referenced until the kernel has run
    dt, dsh, do, dw, dv, ds = (_d(x, cuda) for x in (t, sh, o, w, vis, scr))
    ctx.check(ctx.lib.vs_refine_table(ctx.h, n, ops._ptr(dt), ops._ptr(dsh), 48, 0, ops._ptr(do), ops._ptr(dw),
                                      ops._ptr(dv), ops._ptr(ds), ctypes.byref(cfg), ops._ptr(table)))
    got = table.cpu().numpy()
    assert_bits_equal(got, want, "refine table")
    assert got[:, 0].sum() > 100 and got[:, 1].sum() > 50 and got[:, 3].sum() > 10


@pytest.mark.parametrize("split", [0.0, 0.3])
def test_refine_split_bit_exact(cuda, split):
    n0 = 4000
    t, sh, o, rng = _scene(n0, 2)
    good = np.isfinite(t).all(1) & np.isfinite(sh.reshape(n0, -1)).all(1)
    alive = np.flatnonzero(good)
    parents = np.sort(rng.choice(alive, 600, replace=False)).astype(np.int32)
    dead = np.setdiff1d(np.arange(n0), parents)[:400].astype(np.int32)
    extra = 200
    n = n0 + extra
    children = np.concatenate([dead, np.arange(n0, n)]).astype(np.int32)
    empty = np.setdiff1d(np.arange(n0), np.concatenate([parents, dead]))[:50].astype(np.int32)
    t = np.concatenate([t, np.zeros((extra, 10), np.float32)])
    sh = np.concatenate([sh, np.zeros((extra, 16, 3), np.float32)])
    o = np.concatenate([o, np.zeros(extra, np.float32)])
    scr = (rng.random(n) * 0.9).astype(np.float32)
    wt, wsh, wo = oracle.refine_split(t, sh, o, parents, children, scr, split, MIN_OPACITY, empty)
    ctx = ops.context(cuda)
    dt, dsh, do, dp, dc, ds, de = (_d(x, cuda) for x in (t, sh, o, parents, children, scr, empty))
    ctx.check(ctx.lib.vs_refine_split(ctx.h, n, ops._ptr(dt), ops._ptr(dsh), 48, 0, ops._ptr(do), len(parents),
                                      ops._ptr(dp), ops._ptr(dc), ops._ptr(ds), split, MIN_OPACITY, len(empty),
                                      ops._ptr(de)))
    torch.cuda.synchronize()
    assert_bits_equal(dt.cpu().numpy(), wt, "transforms")
    assert_bits_equal(dsh.cpu().numpy(), wsh, "sh")
    assert_bits_equal(do.cpu().numpy(), wo, "raw opacities")
    # children sit symmetric to their parents about the old mean, with the old SH
    off = wt[children, :3] - t[parents, :3]
    mid_err = np.abs((wt[children, :3] + wt[parents, :3]) / 2 - t[parents, :3])
    assert (mid_err <= 1e-6 * (np.abs(t[parents, :3]) + np.abs(off)) + 1e-7).all()
    assert np.array_equal(wsh[children], sh[parents])


def test_opacity_decay_and_moment_reset(cuda):
    rng = np.random.default_rng(3)
    o = rng.normal(0, 4, 10_000).astype(np.float32)
    ctx = ops.context(cuda)
    do = _d(o, cuda)
    ctx.check(ctx.lib.vs_opacity_decay(ctx.h, o.size, ops._ptr(do), 0.003))
    assert_bits_equal(do.cpu().numpy(), oracle.opacity_decay(o, 0.003), "opacity decay")
    m = ops.Q8Moments(1000 * 48, cuda)
    m.m_codes.random_(0, 256)
    m.v_codes.random_(0, 256)
    before_m, before_v = m.m_codes.clone(), m.v_codes.clone()
    rows = np.array([3, 500, 999, 17], np.int32)
    drows = _d(rows, cuda)
    ctx.check(ctx.lib.vs_q8_reset_rows(ctx.h, m.c(), 48, len(rows), ops._ptr(drows)))
    mc, vc = m.m_codes.view(1000, 48).cpu().numpy(), m.v_codes.view(1000, 48).cpu().numpy()
    assert (mc[rows] == 128).all() and (vc[rows] == 0).all()
    keep = np.setdiff1d(np.arange(1000), rows)
    assert np.array_equal(mc[keep], before_m.view(1000, 48).cpu().numpy()[keep])
    assert np.array_equal(vc[keep], before_v.view(1000, 48).cpu().numpy()[keep])


def test_training_with_refinement(cuda):
    """Config 0 trains, refines (prune + replace + growth toward the cap) and
    keeps training with consistent shapes and finite losses."""
    sp, tgt, cams = scenes.config_tiny()
    cfg_o = oracle.make_cfg(0, mip=True)
    gts = [torch.from_numpy(scenes.pack_rgba8(np.clip(oracle.render_forward(c, cfg_o, tgt)["out_img"][..., :3], 0, 1))
                            .view(np.int32)).to(cuda) for c in cams]
    cfg = TrainConfig(optimizer="q8", total_train_iters=200, refine_every=20, growth_start_iter=0,
                      growth_stop_iter=200, max_splats=30_000, background_noise_strength=0.0)
    tr = SplatTrainer(cfg, cuda, scene_extent=1.0, median_scale=0.02)
    splats = Splats.from_numpy(sp, cuda)
    # a block of splats far too faint to survive: they are pruned and replaced
    with torch.no_grad():
        splats.raw_opacities[:500] = -12.0
    counts, losses = [], []
    for k in range(1, 61):
        splats, st = tr.step(SceneBatch(gts[k % 12], cams[k % 12], k % 12), splats)
        losses.append(float(st.loss.item()))
        if tr.should_refine(k):
            splats, rs = tr.refine(k, splats)
            counts.append((rs.total_splats, rs.num_pruned, rs.num_added))
            n = splats.num_splats
            assert tr.optim["t"].m_codes.numel() == n * 10 and tr.optim["o"].m_codes.numel() == n
            assert tr.optim["sh"].m_codes.numel() == splats.sh_coeffs.numel()
            assert bool(torch.isfinite(splats.transforms).all()) and bool(torch.isfinite(splats.raw_opacities).all())
    assert len(counts) == 3
    assert counts[0][1] >= 500  # the faint block went
    assert counts[-1][0] > sp.n and counts[-1][0] <= 30_000  # grew toward the cap
    assert all(np.isfinite(losses))
