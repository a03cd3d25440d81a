"""View-parallel host logic on two gloo ranks (CPU): the views are partitioned
over the ranks, every rank's dense gradient (computed here by the CPU oracle)
goes through the same exchange layout and all-reduce the GPU path uses, and
the replicated 8-bit Adam step leaves bit-identical replicas equal to a
single-process step over the whole batch."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from vauss_b200.view_parallel import ExchangeLayout, views_for_rank

WORLD = 2
VIEWS_PER_RANK = 2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _scene():
    from vauss_b200 import scenes
    from vauss_b200.camera import look_at
    sp = scenes.random_splats(3000, 5, mean_lo=-1.0, mean_hi=1.0, log_scale_mu=-3.5, log_scale_sigma=0.4,
                              opac_mu=0.0, opac_sigma=1.0, sh_degree=1)
    cams = [look_at((3 * np.cos(a), 3 * np.sin(a), 0.4), (0, 0, 0), 64, 48, 60.0)
            for a in np.linspace(0, 2 * np.pi, 6, endpoint=False)]
    return sp, cams


def _view_grads(sp, cam):
    """Dense gradient rows of one view (oracle render + loss + backward + VJP)."""
    import oracle
    from vauss_b200 import scenes
    cfg = oracle.make_cfg(sp.sh_degree, mip=True)
    r = oracle.render_forward(cam, cfg, sp)
    gt = scenes.pack_rgba8(np.clip(r["out_img"][..., :3] * 0.8 + 0.1, 0, 1))
    lo = oracle.loss_fwd(r["out_img"], gt, 0.8, -0.2)
    dl = oracle.loss_bwd(r["out_img"], gt, lo["coeffs"], 0.8, -0.2)
    vc = oracle.raster_bwd(cam, (0, 0, 0), r["proj"], r["binning_after"], r["out_img"], dl)
    g, _ = oracle.vjp_dense(cam, cfg, sp.transforms, sp.sh, sp.raw_opac, r["proj"]["compact_from_global"], vc)
    return g, r["visible"]


def _adam(sp, grads):
    import oracle
    from vauss_b200 import ops
    n = sp.n
    width = grads.shape[1]
    b1, b2, inv1, inv2 = ops.adam_coefficients(1)
    def zero(c):
        return np.full(c, 128, np.uint8), np.zeros(c, np.uint8), np.zeros((c + 255) // 256, np.float32), \
            np.zeros((c + 255) // 256, np.float32)
    t = oracle.adam_q8(sp.transforms, grads, width, 0, 10, *zero(n * 10), np.float32([1e-3] * 10), 1.0, b1, b2,
                       inv1, inv2, 1e-15, 1)[0]
    wsh = width - 11
    s = oracle.adam_q8(sp.sh.reshape(n, -1), grads, width, 10, wsh, *zero(n * wsh), np.float32([2e-3] * wsh), 1.0,
                       b1, b2, inv1, inv2, 1e-15, 2)[0]
    return np.concatenate([t.reshape(-1), s.reshape(-1)])


def _worker(rank, port, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    sp, cams = _scene()
    width = 10 + sp.sh.shape[1] * 3 + 1
    layout = ExchangeLayout(sp.n, width)
    flat = torch.zeros(layout.size, dtype=torch.float32)
    g, vis = layout.views(flat)
    mine = views_for_rank(len(cams), rank, WORLD, step=1, per_rank=VIEWS_PER_RANK)
    for vi in mine:
        vg, vv = _view_grads(sp, cams[vi])
        g += torch.from_numpy(vg)
        vis += torch.from_numpy(vv)
    dist.all_reduce(flat, op=dist.ReduceOp.SUM)
    params = _adam(sp, g.numpy())
    out_q.put((rank, mine, params, vis.numpy().copy()))
    dist.barrier()
    dist.destroy_process_group()


def test_view_partition_covers_batch():
    for world in (1, 2, 4, 8):
        for step in range(3):
            seen = [v for r in range(world) for v in views_for_rank(200, r, world, step, 1)]
            assert len(set(seen)) == world
            assert seen == [(step * world + r) % 200 for r in range(world)]


def test_two_rank_allreduce_matches_single_process():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in range(WORLD)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    results.sort(key=lambda x: x[0])
    (_, v0, p0, vis0), (_, v1, p1, vis1) = results
    assert set(v0).isdisjoint(v1)
    assert np.array_equal(p0.view(np.uint32), p1.view(np.uint32)), "replicas diverged"
    assert np.array_equal(vis0, vis1)
    # single process: the same views, summed in rank order
    sp, cams = _scene()
    width = 10 + sp.sh.shape[1] * 3 + 1
    total = np.zeros((sp.n, width), np.float32)
    parts = [_view_grads(sp, cams[vi])[0] for vi in v0 + v1]
    per_rank = [parts[0] + parts[1], parts[2] + parts[3]]
    total = per_rank[0] + per_rank[1]
    want = _adam(sp, total)
    np.testing.assert_allclose(p0, want, rtol=0, atol=1e-6)
