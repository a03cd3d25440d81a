"""Compact gradient rows of the view-parallel exchange, checked on one GPU.

A rank that renders one view per step writes compact rows (vs_vjp_compact:
transforms gradient, raw-opacity gradient, colour gradient; 64 bytes) and the
camera position, and the shard owner rebuilds the SH gradient from them
(vs_adam_q8_peer with row_format 1).  Here the ranks are buffers on one
device: each emulated rank renders its own view and writes, from the same
frame and rasterizer gradient, both the dense rows and the compact rows; then
every shard is updated once from the dense rows and once from the compact
rows, starting from the same replicas and moments.  Replicas and moments must
come out bit for bit equal, so the compact exchange inherits the dense
exchange's check against vs_adam_q8_dense (test_gpu_peer.py).

A second view in the same step cannot be represented in a compact row; the
call must report it (VS_ERR_INVALID at the next check), not sum it silently.
"""
import numpy as np
import pytest
import torch

from vauss_b200 import _native as N
from vauss_b200 import ops
from vauss_b200.camera import look_at
from vauss_b200.view_parallel import ViewParallelTrainer
from tests.helpers import assert_bits_equal, medium_scene
from tests.test_gpu_parity import _q8_dev, _q8_host

pytestmark = pytest.mark.gpu


def _np(t):
    return t.detach().cpu().numpy()


def _views(world):
    return [look_at((4.0 * np.cos(a), 4.0 * np.sin(a), 0.8 + 0.3 * k), (0.0, 0.0, 0.0), 250, 170, 220.0)
            for k, a in enumerate(np.linspace(0.3, 2 * np.pi + 0.3, world, endpoint=False))]


@pytest.mark.parametrize("world,deg", [(2, 3), (3, 3), (4, 1)])
def test_compact_rows_update_equals_dense_rows_update(cuda, world, deg):
    sp, _ = medium_scene(sh_degree=deg)
    n, nc = sp.n, (deg + 1) ** 2
    width = 10 + 3 * nc + 1
    dev = cuda
    t, sh, o = (torch.from_numpy(np.ascontiguousarray(x)).to(dev) for x in (sp.transforms, sp.sh, sp.raw_opac))
    cfg = ops.render_cfg(deg, mip=True, background=(0.1, 0.2, 0.3))
    rng = np.random.default_rng(100 * world + deg)
    dense = [torch.zeros(n * width, device=dev) for _ in range(world)]
    compact = [torch.zeros(n * N.COMPACT_ROW, device=dev) for _ in range(world)]
    vis_d = [torch.zeros(n, device=dev) for _ in range(world)]
    vis_c = [torch.zeros(n, device=dev) for _ in range(world)]
    ref_d = [torch.zeros(n, device=dev) for _ in range(world)]
    ref_c = [torch.zeros(n, device=dev) for _ in range(world)]
    cam_c = [torch.zeros(4, device=dev) for _ in range(world)]
    seen = 0
    for r, cam in enumerate(_views(world)):
        out = ops.render(cam, cfg, t, sh, o)
        dl = torch.from_numpy((1e-3 * rng.standard_normal((cam.height, cam.width, 4))).astype(np.float32)).to(dev)
        vc = ops.rasterize_bwd(out.frame, out.out_img, dl)
        ops.vjp_dense(out.frame, cfg, t, sh, o, vc, dense[r], ref_d[r], visible=out.visible, vis_accum=vis_d[r])
        ops.vjp_compact(out.frame, cfg, t, sh, o, vc, compact[r], ref_c[r], cam_c[r], visible=out.visible,
                        vis_accum=vis_c[r])
        seen += out.frame.num_visible
    torch.cuda.synchronize()
    ctx = ops.context(dev)
    assert ctx.lib.vs_ctx_check(ctx.h) == 0
    assert seen > 1000
    for r in range(world):
        assert_bits_equal(_np(vis_c[r]), _np(vis_d[r]), f"view counts of rank {r}")
        assert_bits_equal(_np(ref_c[r]), _np(ref_d[r]), f"refine weights of rank {r}")
        assert _np(cam_c[r])[3] == 0.0

    t0, sh0, o0 = sp.transforms, sp.sh, sp.raw_opac
    mom = dict(t=_q8_host(n * 10, rng), sh=_q8_host(n * nc * 3, rng), o=_q8_host(n, rng))
    lr_t = np.float32([1e-3] * 3 + [2e-3] * 4 + [5e-3] * 3)
    q8 = ops.q8_cfg(5, lr_t, 2.5e-3, 2.5e-4, 5e-2, opac_reg=1e-6, noise_scale=1e-3, noise_limit=0.01,
                    noise_seed=91)
    results = []
    for fmt, rows in ((0, dense), (1, compact)):
        reps = [[torch.from_numpy(np.ascontiguousarray(x).copy()).to(dev) for x in (t0, sh0, o0)]
                for _ in range(world)]
        ps = N.PeerSet()
        ps.world, ps.row_format = world, fmt
        for r in range(world):
            ps.grads[r], ps.vis[r], ps.cams[r] = rows[r].data_ptr(), vis_d[r].data_ptr(), cam_c[r].data_ptr()
            ps.transforms[r], ps.sh_coeffs[r], ps.raw_opacities[r] = (x.data_ptr() for x in reps[r])
        moms = []
        for r in range(world):
            b, e = ViewParallelTrainer.shard_of(n, world, r)
            ps.rank = r
            sm = {}
            for key, per in (("t", 10), ("sh", nc * 3), ("o", 1)):
                h = mom[key]
                sm[key] = _q8_dev(dict(mc=h["mc"][b * per:e * per], vc=h["vc"][b * per:e * per],
                                       ms=h["ms"][b * per // 256:(e * per + 255) // 256],
                                       vs=h["vs"][b * per // 256:(e * per + 255) // 256]), dev)
            ops.adam_q8_peer(deg, n, b, e, ps, sm["t"], sm["sh"], sm["o"], q8, device=dev)
            moms.append(sm)
        torch.cuda.synchronize()
        assert ctx.lib.vs_ctx_check(ctx.h) == 0
        results.append(([[_np(x) for x in rep] for rep in reps], moms))
    (reps_d, moms_d), (reps_c, moms_c) = results
    for r in range(world):
        for k, name in enumerate(("transforms", "sh", "opacity")):
            assert_bits_equal(reps_c[r][k], reps_d[r][k], f"{name} replica {r}")
            assert_bits_equal(reps_c[r][k], reps_d[0][k], f"{name} replica {r} against replica 0")
    assert not np.array_equal(reps_d[0][1], sh0)  # the SH coefficients did move
    for md, mc in zip(moms_d, moms_c):
        for key in ("t", "sh", "o"):
            for f in ("m_codes", "v_codes", "m_scales", "v_scales"):
                assert_bits_equal(_np(getattr(mc[key], f)), _np(getattr(md[key], f)), f"{key} {f}")


def test_second_view_into_compact_rows_is_reported(cuda):
    sp, cams = medium_scene(sh_degree=1)
    n = sp.n
    dev = cuda
    t, sh, o = (torch.from_numpy(np.ascontiguousarray(x)).to(dev) for x in (sp.transforms, sp.sh, sp.raw_opac))
    cfg = ops.render_cfg(1, mip=True)
    rows = torch.zeros(n * N.COMPACT_ROW, device=dev)
    vis, ref, cam = torch.zeros(n, device=dev), torch.zeros(n, device=dev), torch.zeros(4, device=dev)
    ctx = ops.context(dev)
    for k in range(2):
        out = ops.render(cams[0], cfg, t, sh, o)
        dl = torch.full((cams[0].height, cams[0].width, 4), 1e-3, device=dev)
        vc = ops.rasterize_bwd(out.frame, out.out_img, dl)
        ops.vjp_compact(out.frame, cfg, t, sh, o, vc, rows, ref, cam, visible=out.visible, vis_accum=vis)
        torch.cuda.synchronize()
        st = ctx.lib.vs_ctx_check(ctx.h)
        assert st == (0 if k == 0 else 1), ctx.lib.vs_ctx_last_error(ctx.h)  # VS_ERR_INVALID on the second view
    # the error word was cleared
    assert ctx.lib.vs_ctx_check(ctx.h) == 0
