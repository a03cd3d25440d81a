"""Host decisions of the refine step (vauss_b200/refine.py): weighted sampling
without replacement, percentile bounds and the splat budget."""
import numpy as np

from vauss_b200.refine import Bounds, Refiner, weighted_sample
from vauss_b200.trainer import TrainConfig


def test_weighted_sample_distinct_and_weighted():
    rng = np.random.default_rng(0)
    w = np.zeros(1000, np.float32)
    w[:10] = 1.0
    w[10:20] = np.nan
    w[20:30] = -1.0
    got = weighted_sample(rng, w, 50)
    assert sorted(got) == list(range(10))  # only the positive, finite weights, each at most once
    heavy = np.full(1000, 1e-3, np.float32)
    heavy[7] = 1e3
    hits = sum(7 in weighted_sample(np.random.default_rng(s), heavy, 1) for s in range(200))
    assert hits > 190
    assert weighted_sample(rng, np.zeros(5, np.float32), 3) == []


def test_bounds_percentile_and_non_finite():
    rng = np.random.default_rng(1)
    m = rng.uniform(-1, 1, (10_000, 3)).astype(np.float32)
    m[:100] = 1e6  # outliers fall outside the 80 % box
    m[100:110, 1] = np.nan
    b = Bounds.from_means(m)
    assert np.all(np.abs(b.center) < 0.1) and np.all(np.abs(b.extent - 0.8) < 0.05)
    empty = Bounds.from_means(np.full((4, 3), np.nan, np.float32))
    assert np.allclose(empty.extent, 1.0)


def test_splat_cap_follows_the_growth_rate_and_budget():
    c = TrainConfig(total_train_iters=30_000, growth_start_iter=500, growth_stop_iter=2_500)
    r = Refiner(c, Bounds(np.zeros(3, np.float32), np.ones(3, np.float32)), np.random.default_rng(0))
    assert r.splat_cap(100_000) == int(100_000 * 1.05 ** 20.0)  # x1.05 per 100 steps, below the 1.2M budget
    assert r.splat_cap(1_000_000) == 1_200_000
    c.growth_stop_iter = 15_000
    assert r.splat_cap(100_000) == 1_200_000
    assert r.splat_cap(2_000_000) == 2_000_000  # never below the start
    c.max_splats = 777
    assert r.splat_cap(5) == 777
