"""Compact gradient rows of the view-parallel exchange, checked on one GPU.

Each view of a rank's step writes compact rows of its own (vs_vjp_compact:
transforms gradient, raw-opacity gradient, colour gradient; 64 bytes), its bit
in a per-splat view mask and the camera position, and the shard owner
rebuilds the SH gradient from them (vs_adam_q8_peer with row_format 1).  Here
the ranks are buffers on one device and each shard is one launch given all of
them as its peers.  The owner sums over (rank, view) in order, so its update
must equal, bit for bit:

- with one view per rank, the same update from the ranks' dense rows
  (row_format 0, itself checked against vs_adam_q8_dense in test_gpu_peer.py);
- with several views per rank, vs_adam_q8_dense over ONE dense buffer that
  vs_vjp_dense accumulated over the same views in the same order.

A view slot written twice in one step cannot be represented; the call must
report it (VS_ERR_INVALID at the next check), not sum it silently.
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


def _views(count):
    return [look_at((4.0 * np.cos(a), 4.0 * np.sin(a), 0.8 + 0.3 * (k % 3)), (0.0, 0.0, 0.0), 250, 170, 220.0)
            for k, a in enumerate(np.linspace(0.3, 2 * np.pi + 0.3, count, endpoint=False))]


def _shard_moms(mom, n, world, r, nc, dev):
    b, e = ViewParallelTrainer.shard_of(n, world, r)
    sm = {}
    for key, per in (("t", 10), ("sh", nc * 3), ("o", 1)):
        h = mom[key]
        sm[key] = _q8_dev(dict(mc=h["mc"][b * per:e * per], vc=h["vc"][b * per:e * per],
                               ms=h["ms"][b * per // 256:(e * per + 255) // 256],
                               vs=h["vs"][b * per // 256:(e * per + 255) // 256]), dev)
    return b, e, sm


def _peer_update(world, n, deg, nc, params, rows, vis, cams, masks, fmt, views, mom, q8, dev):
    """Every shard updated from the given rows; returns the replicas and the shards' moments."""
    reps = [[torch.from_numpy(np.ascontiguousarray(x).copy()).to(dev) for x in params] for _ in range(world)]
    ps = N.PeerSet()
    ps.world, ps.row_format, ps.views = world, fmt, views
    for r in range(world):
        ps.grads[r], ps.vis[r] = rows[r].data_ptr(), vis[r].data_ptr()
        if fmt == 1:
            ps.cams[r], ps.view_masks[r] = cams[r].data_ptr(), masks[r].data_ptr()
        ps.transforms[r], ps.sh_coeffs[r], ps.raw_opacities[r] = (x.data_ptr() for x in reps[r])
    moms = []
    for r in range(world):
        b, e, sm = _shard_moms(mom, n, world, r, nc, dev)
        ps.rank = r
        ops.adam_q8_peer(deg, n, b, e, ps, sm["t"], sm["sh"], sm["o"], q8, device=dev)
        moms.append((b, e, sm))
    torch.cuda.synchronize()
    return [[_np(x) for x in rep] for rep in reps], moms


@pytest.mark.parametrize("world,views,deg", [(2, 1, 3), (3, 1, 3), (4, 1, 1), (2, 3, 3), (3, 2, 2)])
def test_compact_rows_update(cuda, world, views, deg):
    sp, _ = medium_scene(sh_degree=deg)
    n, nc = sp.n, (deg + 1) ** 2
    width = 10 + 3 * nc + 1
    dev = cuda
    params = (sp.transforms, sp.sh, sp.raw_opac)
    t, sh, o = (torch.from_numpy(np.ascontiguousarray(x)).to(dev) for x in params)
    cfg = ops.render_cfg(deg, mip=True, background=(0.1, 0.2, 0.3))
    rng = np.random.default_rng(100 * world + 10 * views + deg)
    dense = [torch.zeros(n * width, device=dev) for _ in range(world)]        # per rank (one view each)
    flat = torch.zeros(n * width, device=dev)                                  # all views, (rank, view) order
    compact = [torch.zeros(views * n * N.COMPACT_ROW, device=dev) for _ in range(world)]
    vis_d = [torch.zeros(n, device=dev) for _ in range(world)]
    vis_c = [torch.zeros(n, device=dev) for _ in range(world)]
    vis_f = torch.zeros(n, device=dev)
    ref_d, ref_c, ref_f = torch.zeros(n, device=dev), torch.zeros(n, device=dev), torch.zeros(n, device=dev)
    cams = [torch.zeros(views, 4, device=dev) for _ in range(world)]
    masks = [torch.zeros(n, dtype=torch.int32, device=dev) for _ in range(world)]
    cameras = _views(world * views)
    seen = 0
    for r in range(world):
        for v in range(views):
            cam = cameras[r * views + v]
            out = ops.render(cam, cfg, t, sh, o)
            dl = torch.from_numpy((1e-3 * rng.standard_normal((cam.height, cam.width, 4))).astype(np.float32)).to(dev)
            vc = ops.rasterize_bwd(out.frame, out.out_img, dl)
            if views == 1:
                ops.vjp_dense(out.frame, cfg, t, sh, o, vc, dense[r], ref_d, visible=out.visible, vis_accum=vis_d[r])
            ops.vjp_dense(out.frame, cfg, t, sh, o, vc, flat, ref_f, visible=out.visible, vis_accum=vis_f)
            rows = compact[r][v * n * N.COMPACT_ROW:(v + 1) * n * N.COMPACT_ROW]
            ops.vjp_compact(out.frame, cfg, t, sh, o, vc, rows, ref_c, cams[r][v], masks[r], v, visible=out.visible,
                            vis_accum=vis_c[r])
            seen += out.frame.num_visible
    torch.cuda.synchronize()
    ctx = ops.context(dev)
    assert ctx.lib.vs_ctx_check(ctx.h) == 0
    assert seen > 1000
    assert_bits_equal(_np(ref_c), _np(ref_f), "refine weights")
    assert_bits_equal(_np(sum(vis_c[1:], vis_c[0].clone()) if world > 1 else vis_c[0]), _np(vis_f), "view counts")
    for r in range(world):
        assert (_np(masks[r]) >> views == 0).all() and _np(cams[r])[:, 3].max() == 0.0

    mom = dict(t=_q8_host(n * 10, rng), sh=_q8_host(n * nc * 3, rng), o=_q8_host(n, rng))
    lr_t = np.float32([1e-3] * 3 + [2e-3] * 4 + [5e-3] * 3)
    q8 = ops.q8_cfg(5, lr_t, 2.5e-3, 2.5e-4, 5e-2, opac_reg=1e-6, noise_scale=1e-3, noise_limit=0.01,
                    noise_seed=91)
    reps_c, moms_c = _peer_update(world, n, deg, nc, params, compact, vis_c, cams, masks, 1, views, mom, q8, dev)
    if views == 1:
        want_reps, want_moms = _peer_update(world, n, deg, nc, params, dense, vis_d, None, None, 0, 0, mom, q8, dev)
        want = want_reps[0]
    else:
        dt, dsh, do = (torch.from_numpy(np.ascontiguousarray(x).copy()).to(dev) for x in params)
        dm = {k: _q8_dev(v, dev) for k, v in mom.items()}
        ops.adam_q8_dense(deg, dt, dsh, do, flat.view(n, width), dm["t"], dm["sh"], dm["o"], q8, visible=vis_f)
        torch.cuda.synchronize()
        want = [_np(dt), _np(dsh), _np(do)]
        want_moms = None
    assert ctx.lib.vs_ctx_check(ctx.h) == 0
    for r in range(world):
        for k, name in enumerate(("transforms", "sh", "opacity")):
            assert_bits_equal(reps_c[r][k], want[k], f"{name} replica {r}")
    assert not np.array_equal(want[1], sp.sh)  # the SH coefficients did move
    for i, (b, e, sm) in enumerate(moms_c):
        for key, per in (("t", 10), ("sh", nc * 3), ("o", 1)):
            for f in ("m_codes", "v_codes", "m_scales", "v_scales"):
                got = _np(getattr(sm[key], f))
                if want_moms is not None:
                    ref = _np(getattr(want_moms[i][2][key], f))
                else:
                    full = _np(getattr(dm[key], f))
                    ref = full[b * per:e * per] if f.endswith("codes") else full[b * per // 256:b * per // 256 + got.size]
                assert_bits_equal(got, ref, f"{key} {f} shard {i}")


def test_view_slot_written_twice_is_reported(cuda):
    sp, cams = medium_scene(sh_degree=1)
    n = sp.n
    dev = cuda
    t, sh, o = (torch.from_numpy(np.ascontiguousarray(x)).to(dev) for x in (sp.transforms, sp.sh, sp.raw_opac))
    cfg = ops.render_cfg(1, mip=True)
    rows = torch.zeros(n * N.COMPACT_ROW, device=dev)
    vis, ref, cam = torch.zeros(n, device=dev), torch.zeros(n, device=dev), torch.zeros(4, device=dev)
    mask = torch.zeros(n, dtype=torch.int32, device=dev)
    ctx = ops.context(dev)
    for k in range(2):
        out = ops.render(cams[0], cfg, t, sh, o)
        dl = torch.full((cams[0].height, cams[0].width, 4), 1e-3, device=dev)
        vc = ops.rasterize_bwd(out.frame, out.out_img, dl)
        ops.vjp_compact(out.frame, cfg, t, sh, o, vc, rows, ref, cam, mask, 0, visible=out.visible, vis_accum=vis)
        torch.cuda.synchronize()
        st = ctx.lib.vs_ctx_check(ctx.h)
        assert st == (0 if k == 0 else 1), ctx.lib.vs_ctx_last_error(ctx.h)  # VS_ERR_INVALID on the reuse
    assert ctx.lib.vs_ctx_check(ctx.h) == 0  # the error word was cleared
    assert int(_np(mask).max()) == 1
