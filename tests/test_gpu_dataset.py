"""The dataset feed on the GPU: the packing kernel against the oracle for
every source layout, and the staged loader (vs_feed_*) in streaming and
HBM-cached modes against the oracle's packing of the views it reports, in
the order vs_feed_order gives."""
import numpy as np
import pytest
import torch

import oracle
from vauss_b200 import _native, dataset, scenes
from vauss_b200.trainer import Splats, SplatTrainer, TrainConfig

pytestmark = pytest.mark.gpu


def _img(rng, h, w, c):
    return rng.integers(0, 256, (h, w, c), dtype=np.uint8)


@pytest.mark.parametrize("c", [1, 2, 3, 4])
@pytest.mark.parametrize("mode", [dataset.AlphaMode.MASKED, dataset.AlphaMode.TRANSPARENT])
@pytest.mark.parametrize("hw", [(1, 1), (3, 5), (37, 23), (256, 301)])
def test_pack_view_matches_oracle(cuda, c, mode, hw):
    img = _img(np.random.default_rng(c * 100 + hw[0]), hw[0], hw[1], c)
    got, has_alpha = dataset.view_to_packed_data(img, mode, cuda)
    want, want_alpha = oracle.pack_view(img, int(mode))
    assert has_alpha == want_alpha
    np.testing.assert_array_equal(got.cpu().numpy().view(np.uint32), want)


def _views(rng, sizes):
    return [dataset.SceneView(_img(rng, h, w, c), None, mode) for (h, w, c, mode) in sizes]


SIZES = [(64, 80, 3, 0), (33, 17, 4, 1), (128, 96, 4, 0), (5, 7, 1, 0), (40, 41, 2, 1), (64, 80, 3, 0)]


@pytest.mark.parametrize("ring", [2, 4])
def test_streaming_feed_order_and_content(cuda, ring):
    views = _views(np.random.default_rng(ring), SIZES)
    want = [oracle.pack_view(v.image, int(v.alpha_mode))[0] for v in views]
    loader = dataset.SceneLoader(dataset.Scene(views), seed=99, device=cuda,
                                 config=dataset.LoadDatasetConfig(max_scene_batch_cache_size=0), ring_slots=ring)
    order = dataset.visiting_order(99, len(views), 4 * len(views))
    sums = []
    for k, vi in enumerate(order):
        b = loader.next_batch()
        assert b.view_index == vi and not loader.last_cached
        assert loader.last_h2d_bytes == views[vi].image.size
        assert b.has_alpha == (views[vi].image.shape[2] in (2, 4))
        # device work on the batch in stream order, read back later: a slot
        # rewritten too early would change the result
        sums.append((vi, b.img_packed.to(torch.int64).sum(), b.img_packed.clone()))
    torch.cuda.synchronize()
    for vi, s, copy in sums:
        np.testing.assert_array_equal(copy.cpu().numpy().view(np.uint32), want[vi])
        assert int(s.item()) == int(want[vi].view(np.int32).astype(np.int64).sum())
    loader.close()


@pytest.mark.parametrize("hold", [2, 3])
def test_streaming_feed_holds_several_batches(cuda, hold):
    """A step that uses `hold` batches at once reads each only after taking
    all of them; none may be overwritten by the staging of later ones."""
    views = _views(np.random.default_rng(11 + hold), SIZES)
    want = [oracle.pack_view(v.image, int(v.alpha_mode))[0] for v in views]
    loader = dataset.SceneLoader(dataset.Scene(views), seed=5, device=cuda, ring_slots=2, hold=hold,
                                 config=dataset.LoadDatasetConfig(max_scene_batch_cache_size=0))
    got = []
    for step in range(8):
        batches = [loader.next_batch() for _ in range(hold)]
        got += [(b.view_index, b.img_packed.clone()) for b in batches]
    torch.cuda.synchronize()
    for vi, img in got:
        np.testing.assert_array_equal(img.cpu().numpy().view(np.uint32), want[vi])
    loader.close()


def test_cached_feed_copies_each_view_once(cuda):
    views = _views(np.random.default_rng(5), SIZES)
    want = [oracle.pack_view(v.image, int(v.alpha_mode))[0] for v in views]
    loader = dataset.SceneLoader(dataset.Scene(views), seed=3, device=cuda, ring_slots=3)
    n = len(views)
    h2d = []
    for k in range(3 * n):
        b = loader.next_batch()
        h2d.append(loader.last_h2d_bytes)
        np.testing.assert_array_equal(b.img_packed.cpu().numpy().view(np.uint32), want[b.view_index])
        assert loader.last_cached
    assert sum(h2d) == sum(v.image.size for v in views)  # each view crossed once
    loader.close()


def test_cache_budget_admits_only_what_fits(cuda):
    rng = np.random.default_rng(8)
    views = [dataset.SceneView(_img(rng, 32, 32, 3), None) for _ in range(5)]
    budget = int(2.5 * 32 * 32 * 4)  # two packed views fit
    loader = dataset.SceneLoader(dataset.Scene(views), seed=1, device=cuda, ring_slots=2,
                                 config=dataset.LoadDatasetConfig(max_scene_batch_cache_size=budget))
    cached_views = set()
    for _ in range(4 * 5):
        b = loader.next_batch()
        if loader.last_cached:
            cached_views.add(b.view_index)
        np.testing.assert_array_equal(b.img_packed.cpu().numpy().view(np.uint32),
                                      oracle.pack_view(views[b.view_index].image)[0])
    assert len(cached_views) == 2
    loader.close()


def test_feed_argument_errors(cuda):
    from vauss_b200 import ops
    import ctypes
    ctx = ops.context(cuda)
    c = _native.FeedCfg()
    c.num_views, c.ring_slots = 2, 1
    h = ctypes.c_void_p()
    assert ctx.lib.vs_feed_create(ctx.h, ctypes.byref(c), ctypes.byref(h)) == 1
    c.ring_slots = 2
    assert ctx.lib.vs_feed_create(ctx.h, ctypes.byref(c), ctypes.byref(h)) == 1  # hold 0
    c.hold = 1
    ctx.check(ctx.lib.vs_feed_create(ctx.h, ctypes.byref(c), ctypes.byref(h)))
    px = np.zeros((4, 4, 3), np.uint8)
    assert ctx.lib.vs_feed_set_view(h, 0, px.ctypes.data, 4, 4, 5, 0) == 1
    ctx.check(ctx.lib.vs_feed_set_view(h, 0, px.ctypes.data, 4, 4, 3, 0))
    b = _native.SceneBatchC()
    assert ctx.lib.vs_feed_next(h, ctypes.byref(b)) == 1  # view 1 never set
    assert b"never set" in ctx.lib.vs_ctx_last_error(ctx.h)
    ctx.lib.vs_feed_destroy(h)


def test_training_from_the_feed(cuda):
    """Config 0 trains from the staged loader (RGB sources): the packed
    ground truth equals the scenes' own packing and the loss falls."""
    sp, tgt, cams = scenes.config_tiny()
    cfg_o = oracle.make_cfg(0, mip=True)
    packed = [scenes.pack_rgba8(np.clip(oracle.render_forward(c, cfg_o, tgt)["out_img"][..., :3], 0, 1))
              for c in cams]
    rgb = [p.view(np.uint8).reshape(p.shape[0], p.shape[1], 4)[..., :3].copy() for p in packed]
    views = [dataset.SceneView(img, cam) for img, cam in zip(rgb, cams)]
    loader = dataset.SceneLoader(dataset.Scene(views), seed=7, device=cuda,
                                 config=dataset.LoadDatasetConfig(max_scene_batch_cache_size=0))
    cfg = TrainConfig(optimizer="q8", total_train_iters=100, lr_mean=1e-3, lr_mean_end=1e-3, lr_scale=5e-3,
                      lr_opac=5e-2, lr_coeffs_dc=2.5e-3, background_noise_strength=0.0)
    tr = SplatTrainer(cfg, cuda, scene_extent=1.0, median_scale=0.02)
    splats = Splats.from_numpy(sp, cuda)
    losses = []
    for k in range(96):
        b = loader.next_batch()
        if k < 12:
            np.testing.assert_array_equal(b.img_packed.cpu().numpy().view(np.uint32), packed[b.view_index])
        splats, st = tr.step(b, splats)
        losses.append(float(st.loss.item()))
    assert np.mean(losses[-12:]) < np.mean(losses[:12])
    loader.close()
