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
