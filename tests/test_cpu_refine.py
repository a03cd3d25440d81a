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


def test_oracle_min_scale_and_fold_against_float64():
    """The oracle's 3D-filter floor and bake against a float64 restatement of
    compute_min_scale (train.rs:353-387) and fold_min_scale
    (gaussian_splats.rs:165-188)."""
    import oracle
    rng = np.random.default_rng(4)
    n, v = 3000, 7
    t = np.zeros((n, 10), np.float32)
    t[:, :3] = rng.uniform(-2, 2, (n, 3))
    t[:, 7:10] = rng.normal(-4, 1, (n, 3))
    raw = rng.normal(0, 2, n).astype(np.float32)
    centres = rng.uniform(-5, 5, (v, 3)).astype(np.float32)
    focal = rng.uniform(200, 2000, v).astype(np.float32)
    rows = np.concatenate([centres, (1.0 / np.maximum(focal, 1e-6)).astype(np.float32)[:, None]], 1).astype(np.float32)
    got = oracle.min_scale(t, rows, 0.1)
    d = np.linalg.norm(t[:, None, :3].astype(np.float64) - centres[None].astype(np.float64), axis=2)
    want = np.sqrt(0.1) * (d / focal[None].astype(np.float64)).min(axis=1)
    np.testing.assert_allclose(got, want, rtol=2e-6)
    ms = (got * 40).astype(np.float32)
    ft, fo = oracle.fold_min_scale(t, raw, ms)
    s = np.exp(t[:, 7:10].astype(np.float64))
    new_log = 0.5 * np.log(s * s + ms[:, None].astype(np.float64) ** 2)
    np.testing.assert_allclose(ft[:, 7:10], new_log, rtol=1e-5, atol=1e-5)
    coef = np.exp((t[:, 7:10] - new_log).sum(axis=1))
    o = np.clip(1.0 / (1.0 + np.exp(-raw.astype(np.float64))) * coef, 1e-6, 1 - 1e-6)
    np.testing.assert_allclose(fo, np.log(o / (1 - o)), rtol=1e-4, atol=2e-4)
    np.testing.assert_array_equal(ft[:, :7], t[:, :7])
