"""The view-parallel exchange over peer memory, checked on one GPU.

vs_adam_q8_peer is the sharded optimizer of the multi-GPU step: each rank
updates its shard of the splats from the gradient rows of every rank (read
over NVLink) and stores the result into every replica.  Here the "ranks" are
buffers on one device, and each shard is one launch given all of them as its
peers; the launches run one after another, so nothing waits on anything.  The
result must equal vs_adam_q8_dense (itself checked against the oracle) applied
to the rank-order sum of the rows of the ranks that saw each splat.

The device barrier's bounded wait is checked by making it run out: a flag
that nothing sets must give VS_ERR_DEVICE_TIMEOUT, not a hang or a fault.
"""
import ctypes
import time

import numpy as np
import pytest
import torch

from vauss_b200 import _native as N
from vauss_b200 import ops
from vauss_b200.view_parallel import ViewParallelTrainer
from tests.helpers import assert_bits_equal
from tests.test_gpu_parity import _q8_dev, _q8_host

pytestmark = pytest.mark.gpu


def _np(t):
    return t.detach().cpu().numpy()


@pytest.mark.parametrize("world,n", [(3, 2_000), (2, 513), (4, 256 * 5 + 3)])
def test_sharded_peer_adam_matches_dense(cuda, world, n):
    rng = np.random.default_rng(world * 1000 + n)
    deg, nc = 3, 16
    width = 10 + nc * 3 + 1
    t0 = rng.standard_normal((n, 10)).astype(np.float32)
    sh0 = (0.3 * rng.standard_normal((n, nc, 3))).astype(np.float32)
    o0 = rng.standard_normal(n).astype(np.float32)
    grads = [(1e-3 * rng.standard_normal((n, width))).astype(np.float32) for _ in range(world)]
    vis = [rng.integers(0, 3, size=n).astype(np.float32) * (rng.random(n) < 0.6) for _ in range(world)]
    for r in range(world):  # rows of ranks that did not see a splat hold stale values: they must be skipped
        grads[r][vis[r] == 0] = 1e3
    mom = dict(t=_q8_host(n * 10, rng), sh=_q8_host(n * nc * 3, rng), o=_q8_host(n, rng))
    lr_t = np.float32([1e-3] * 3 + [2e-3] * 4 + [5e-3] * 3)
    q8 = ops.q8_cfg(4, lr_t, 2.5e-3, 2.5e-4, 5e-2, opac_reg=1e-6, noise_scale=1e-3, noise_limit=0.01,
                    noise_seed=77)

    # dense reference: rank-order sum of the rows with vis > 0
    gsum = np.zeros((n, width), np.float32)
    vsum = np.zeros(n, np.float32)
    for r in range(world):
        gsum = gsum + np.where((vis[r] > 0)[:, None], grads[r], np.float32(0))
        vsum = vsum + vis[r]
    dt, dsh, do = (torch.from_numpy(x.copy()).to(cuda) for x in (t0, sh0, o0))
    dm = {k: _q8_dev(v, cuda) for k, v in mom.items()}
    ops.adam_q8_dense(deg, dt, dsh, do, torch.from_numpy(gsum).to(cuda), dm["t"], dm["sh"], dm["o"], q8,
                      visible=torch.from_numpy(vsum).to(cuda))

    # sharded over `world` emulated ranks
    reps = [[torch.from_numpy(x.copy()).to(cuda) for x in (t0, sh0, o0)] for _ in range(world)]
    g_dev = [torch.from_numpy(g).to(cuda) for g in grads]
    v_dev = [torch.from_numpy(v).to(cuda) for v in vis]
    ps = N.PeerSet()
    ps.world = world
    for r in range(world):
        ps.grads[r], ps.vis[r] = g_dev[r].data_ptr(), v_dev[r].data_ptr()
        ps.transforms[r], ps.sh_coeffs[r], ps.raw_opacities[r] = (x.data_ptr() for x in reps[r])
    shard_moms = []
    for r in range(world):
        b, e = ViewParallelTrainer.shard_of(n, world, r)
        ps.rank = r
        sm = {}
        for key, per in (("t", 10), ("sh", nc * 3), ("o", 1)):
            h = mom[key]
            sm[key] = _q8_dev(dict(mc=h["mc"][b * per:e * per], vc=h["vc"][b * per:e * per],
                                   ms=h["ms"][b * per // 256:(e * per + 255) // 256],
                                   vs=h["vs"][b * per // 256:(e * per + 255) // 256]), cuda)
        ops.adam_q8_peer(deg, n, b, e, ps, sm["t"], sm["sh"], sm["o"], q8, device=cuda)
        shard_moms.append((b, e, sm))
    torch.cuda.synchronize()
    for r in range(world):
        assert_bits_equal(_np(reps[r][0]), _np(dt), f"transforms replica {r}")
        assert_bits_equal(_np(reps[r][1]), _np(dsh), f"sh replica {r}")
        assert_bits_equal(_np(reps[r][2]), _np(do), f"opacity replica {r}")
    for b, e, sm in shard_moms:
        for key, per in (("t", 10), ("sh", nc * 3), ("o", 1)):
            full = dm[key]
            assert_bits_equal(_np(sm[key].m_codes), _np(full.m_codes)[b * per:e * per], f"{key} m codes")
            assert_bits_equal(_np(sm[key].v_codes), _np(full.v_codes)[b * per:e * per], f"{key} v codes")
            nb = sm[key].m_scales.numel()
            assert_bits_equal(_np(sm[key].m_scales), _np(full.m_scales)[b * per // 256:b * per // 256 + nb],
                              f"{key} m scales")
            assert_bits_equal(_np(sm[key].v_scales), _np(full.v_scales)[b * per // 256:b * per // 256 + nb],
                              f"{key} v scales")


def test_shards_cover_every_block_once():
    for n in (1, 255, 256, 257, 3_000_000):
        for world in (1, 2, 3, 8):
            spans = [ViewParallelTrainer.shard_of(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            for (b0, e0), (b1, e1) in zip(spans, spans[1:]):
                assert e0 == b1 and b0 % 256 == 0 and b1 % 256 == 0


def _flags(cuda, *vals):
    return torch.tensor(list(vals), dtype=torch.int32, device=cuda)


def _barrier(ctx, flag_tensors, world, rank, epoch):
    ptrs = (ctypes.c_void_p * N.PEER_MAX)(*[f.data_ptr() for f in flag_tensors])
    return ctx.lib.vs_peer_barrier(ctx.h, ptrs, world, rank, epoch)


def test_barrier_passes_when_every_rank_has_signalled(cuda):
    ctx = ops.context(cuda)
    mine, other = _flags(cuda, 0, 7), _flags(cuda, 0, 0)  # rank 1 already stored epoch 7 into our slot
    assert _barrier(ctx, [mine, other], 2, 0, 7) == 0
    assert ctx.lib.vs_ctx_check(ctx.h) == 0
    assert int(mine[0]) == 7 and int(other[0]) == 7  # our signal reached both arrays


def test_barrier_wait_runs_out_with_an_error(cuda):
    ctx = ops.context(cuda)
    mine, other = _flags(cuda, 0, 0), _flags(cuda, 0, 0)  # nobody signals slot 1
    t = time.time()
    assert _barrier(ctx, [mine, other], 2, 0, 1) == 0  # the launch itself is fine
    st = ctx.lib.vs_ctx_check(ctx.h)
    assert st == 4, ctx.lib.vs_ctx_last_error(ctx.h)  # VS_ERR_DEVICE_TIMEOUT
    assert time.time() - t < 60
    # the context stays usable, and the error word was cleared
    assert _barrier(ctx, [mine], 1, 0, 2) == 0
    assert ctx.lib.vs_ctx_check(ctx.h) == 0


def test_peer_adam_after_a_barrier_that_gave_up_touches_nothing(cuda):
    """A barrier whose wait ran out leaves VS_DERR_WAIT in the device error
    word; the sharded update launched after it must then neither read the
    peers' (possibly incomplete) rows nor store into any replica."""
    world, n, nc = 2, 700, 16
    width = 10 + nc * 3 + 1
    rng = np.random.default_rng(31)
    t0 = rng.standard_normal((n, 10)).astype(np.float32)
    sh0 = (0.3 * rng.standard_normal((n, nc, 3))).astype(np.float32)
    o0 = rng.standard_normal(n).astype(np.float32)
    reps = [[torch.from_numpy(x.copy()).to(cuda) for x in (t0, sh0, o0)] for _ in range(world)]
    g_dev = [torch.from_numpy((1e-3 * rng.standard_normal((n, width))).astype(np.float32)).to(cuda)
             for _ in range(world)]
    v_dev = [torch.ones(n, device=cuda) for _ in range(world)]
    ps = N.PeerSet()
    ps.world, ps.rank = world, 0
    for r in range(world):
        ps.grads[r], ps.vis[r] = g_dev[r].data_ptr(), v_dev[r].data_ptr()
        ps.transforms[r], ps.sh_coeffs[r], ps.raw_opacities[r] = (x.data_ptr() for x in reps[r])
    b, e = ViewParallelTrainer.shard_of(n, world, 0)
    mom = {k: _q8_host(c, rng) for k, c in (("t", (e - b) * 10), ("sh", (e - b) * nc * 3), ("o", e - b))}
    dm = {k: _q8_dev(v, cuda) for k, v in mom.items()}
    q8 = ops.q8_cfg(3, np.float32([1e-3] * 10), 2.5e-3, 2.5e-4, 5e-2)
    ctx = ops.context(cuda)
    mine, other = _flags(cuda, 0, 0), _flags(cuda, 0, 0)  # rank 1 never signals
    assert _barrier(ctx, [mine, other], world, 0, 1) == 0
    ops.adam_q8_peer(3, n, b, e, ps, dm["t"], dm["sh"], dm["o"], q8, device=cuda)
    torch.cuda.synchronize()
    for r in range(world):
        assert_bits_equal(_np(reps[r][0]), t0, f"transforms replica {r}")
        assert_bits_equal(_np(reps[r][1]), sh0, f"sh replica {r}")
        assert_bits_equal(_np(reps[r][2]), o0, f"opacity replica {r}")
    for k, h in mom.items():
        assert_bits_equal(_np(dm[k].m_codes), h["mc"], f"{k} m codes")
        assert_bits_equal(_np(dm[k].v_scales), h["vs"], f"{k} v scales")
    assert ctx.lib.vs_ctx_check(ctx.h) == 4  # VS_ERR_DEVICE_TIMEOUT, and the word is cleared
    # with the word clear, the same launch updates the replicas again
    ops.adam_q8_peer(3, n, b, e, ps, dm["t"], dm["sh"], dm["o"], q8, device=cuda)
    torch.cuda.synchronize()
    assert not np.array_equal(_np(reps[1][0])[:e], t0[:e])
    assert ctx.lib.vs_ctx_check(ctx.h) == 0


@pytest.mark.parametrize("world,views", [(2, 2), (3, 1), (1, 3)])
def test_owner_vjp_exchange_matches_dense_exchange(cuda, world, views):
    """The owner-side exchange (vs_vjp_owner + vs_adam_q8_shard: each shard's
    owner computes the projection VJP of every rank's views from the views'
    maps, visible marks, rasterizer rows and uniforms) against the dense one
    (vs_vjp_dense on every rank, then vs_adam_q8_peer): the owner's rows equal
    the rank-order sums of the dense rows, and both give the same replicas and
    moments bit for bit.  Ranks are emulated on one device; the rasterizer rows
    are random, including rows of splats whose visible mark is 0."""
    from vauss_b200.camera import look_at
    from tests.helpers import medium_scene
    sp, _ = medium_scene(seed=70 + world, n=4000)
    n, nc = sp.n, sp.sh.shape[1]
    width = 10 + nc * 3 + 1
    cfg = ops.render_cfg(3, mip=True)
    rng = np.random.default_rng(world * 10 + views)
    t0, sh0, o0 = (torch.from_numpy(x).to(cuda) for x in (sp.transforms, sp.sh, sp.raw_opac))
    vs = N.ViewSet()
    vs.world = world
    dense_rows, dense_vis, keep = [], [], []
    for r in range(world):
        g_r = torch.zeros(n, width, device=cuda)
        v_r = torch.zeros(n, device=cuda)
        refine = torch.zeros(n, device=cuda)
        for k in range(views):
            a = rng.uniform(0, 2 * np.pi)
            cam = look_at((4.0 * np.cos(a), 4.0 * np.sin(a), rng.uniform(-1, 1)), (0, 0, 0), 250, 170, 220.0)
            out = ops.render(cam, cfg, t0, sh0, o0)
            nv = out.num_visible
            vc = torch.zeros(n, 10, device=cuda)
            rows_h = (1e-3 * rng.standard_normal((nv, 10))).astype(np.float32)
            rows_h[rng.random(nv) < 0.2] = 0.0
            vc[:nv] = torch.from_numpy(rows_h).to(cuda)
            ops.vjp_dense(out.frame, cfg, t0, sh0, o0, vc[:max(nv, 1)], g_r, refine, visible=out.visible,
                          vis_accum=v_r)
            cmap = torch.empty(n, dtype=torch.int32, device=cuda)
            out.frame.copy_field("compact_from_global", cmap)
            uni = torch.zeros(N.UNIFORMS_BYTES // 4, dtype=torch.int32, device=cuda)
            ops.frame_uniforms(out.frame, uni)
            j = r * N.VIEW_SLOTS + k
            vs.compact_from_global[j], vs.visible[j] = cmap.data_ptr(), out.visible.data_ptr()
            vs.v_combined[j], vs.uniforms[j] = vc.data_ptr(), uni.data_ptr()
            keep += [out, vc, cmap, uni]
        vs.used[r] = views
        dense_rows.append(g_r)
        dense_vis.append(v_r)
    torch.cuda.synchronize()
    lr_t = np.float32([1e-3] * 3 + [2e-3] * 4 + [5e-3] * 3)
    q8 = ops.q8_cfg(3, lr_t, 2.5e-3, 2.5e-4, 5e-2, opac_reg=1e-6, noise_scale=1e-3, noise_limit=0.01, noise_seed=5)
    mom_h = dict(t=_q8_host(n * 10, rng), sh=_q8_host(n * nc * 3, rng), o=_q8_host(n, rng))

    def replicas():
        return [[x.clone() for x in (t0, sh0, o0)] for _ in range(world)]

    def peer_set(reps, rows=None, vis=None):
        ps = N.PeerSet()
        ps.world = world
        for r in range(world):
            ps.transforms[r], ps.sh_coeffs[r], ps.raw_opacities[r] = (x.data_ptr() for x in reps[r])
            if rows is not None:
                ps.grads[r], ps.vis[r] = rows[r].data_ptr(), vis[r].data_ptr()
        return ps

    def shard_moms(b, e):
        out = {}
        for key, per in (("t", 10), ("sh", nc * 3), ("o", 1)):
            h = mom_h[key]
            out[key] = _q8_dev(dict(mc=h["mc"][b * per:e * per], vc=h["vc"][b * per:e * per],
                                    ms=h["ms"][b * per // 256:(e * per + 255) // 256],
                                    vs=h["vs"][b * per // 256:(e * per + 255) // 256]), cuda)
        return out

    rep_d, rep_o = replicas(), replicas()
    ps_d, ps_o = peer_set(rep_d, dense_rows, dense_vis), peer_set(rep_o)
    moms_d, moms_o = [], []
    for r in range(world):
        b, e = ViewParallelTrainer.shard_of(n, world, r)
        ps_d.rank = ps_o.rank = r
        md, mo = shard_moms(b, e), shard_moms(b, e)
        ops.adam_q8_peer(3, n, b, e, ps_d, md["t"], md["sh"], md["o"], q8, device=cuda)
        rows = torch.zeros(max(e - b, 1), width, device=cuda)
        vis = torch.zeros(max(e - b, 1), device=cuda)
        ops.vjp_owner(3, n, b, e, vs, t0, sh0, o0, rows, vis, device=cuda)
        ops.adam_q8_shard(3, n, b, e, rows, vis, ps_o, mo["t"], mo["sh"], mo["o"], q8, device=cuda)
        torch.cuda.synchronize()
        # rows: the rank-order sum of the dense rows of the ranks that saw the splat
        want_vis = np.zeros(e - b, np.float32)
        want = np.zeros((e - b, width), np.float32)
        for v_r, g_r in zip(dense_vis, dense_rows):
            want_vis = (want_vis + _np(v_r)[b:e]).astype(np.float32)
            want = np.where((_np(v_r)[b:e] > 0)[:, None], want + _np(g_r)[b:e], want).astype(np.float32)
        seen = want_vis > 0
        assert_bits_equal(_np(vis)[:e - b], want_vis, f"view counts of shard {r}")
        assert_bits_equal(_np(rows)[:e - b][seen], want[seen], f"rows of shard {r}")
        moms_d.append(md)
        moms_o.append(mo)
    for r in range(world):
        for i, name in enumerate(("transforms", "sh", "opacity")):
            assert_bits_equal(_np(rep_o[r][i]), _np(rep_d[r][i]), f"{name} replica {r}")
    for md, mo in zip(moms_d, moms_o):
        for key in ("t", "sh", "o"):
            assert_bits_equal(_np(mo[key].m_codes), _np(md[key].m_codes), f"{key} m codes")
            assert_bits_equal(_np(mo[key].v_scales), _np(md[key].v_scales), f"{key} v scales")
