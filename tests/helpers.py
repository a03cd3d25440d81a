"""Shared scene builders and comparison helpers for the tests."""
from __future__ import annotations

import numpy as np

from vauss_b200 import scenes
from vauss_b200.camera import look_at

# Tolerance for floating-point outputs whose summation order differs between
# the GPU and the oracle (atomics in the rasterizer backward): 1e-4 relative,
# with an absolute floor proportional to the tensor's scale (near-zero lanes).
REL_TOL = 1e-4


def medium_scene(seed: int = 7, n: int = 40_000, sh_degree: int = 3):
    """SH-3 splats in [-1.5, 1.5]^3 seen by two cameras of 250x170 (partial
    edge tiles in both directions)."""
    sp = scenes.random_splats(n, seed, mean_lo=-1.5, mean_hi=1.5, log_scale_mu=-3.8, log_scale_sigma=0.6,
                              opac_mu=0.0, opac_sigma=1.5, sh_degree=sh_degree)
    cams = [look_at((4.0, 0.3, 0.6), (0, 0, 0), 250, 170, 220.0),
            look_at((-2.5, 3.0, -0.8), (0.1, 0, 0), 250, 170, 260.0)]
    return sp, cams


def tiny_scene():
    sp, tgt, cams = scenes.config_tiny()
    return sp, tgt, cams


def assert_mixed_close(got, want, rel=REL_TOL, floor_frac=1e-3, what=""):
    """|got - want| <= rel * max(|want|, s), s = floor_frac * max|want| of the tensor."""
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    assert got.shape == want.shape, f"{what}: shape {got.shape} != {want.shape}"
    scale = floor_frac * max(float(np.abs(want).max()) if want.size else 0.0, 1e-30)
    bound = rel * np.maximum(np.abs(want), scale)
    err = np.abs(got - want)
    bad = err > bound
    if bad.any():
        i = np.unravel_index(np.argmax(err - bound), err.shape)
        raise AssertionError(f"{what}: {int(bad.sum())}/{bad.size} out of tolerance; worst at {i}: "
                             f"got {got[i]!r} want {want[i]!r} (bound {bound[i]:.3g})")


def assert_bits_equal(got, want, what=""):
    got = np.ascontiguousarray(got)
    want = np.ascontiguousarray(want)
    assert got.shape == want.shape, f"{what}: shape {got.shape} != {want.shape}"
    gv = got.view(np.uint32) if got.dtype.itemsize == 4 else got
    wv = want.view(np.uint32) if want.dtype.itemsize == 4 else want
    bad = gv != wv
    if bad.any():
        idx = np.argwhere(bad)[:5]
        raise AssertionError(f"{what}: {int(bad.sum())}/{bad.size} differ; first {idx.tolist()}: "
                             f"got {[got[tuple(j)] for j in idx]} want {[want[tuple(j)] for j in idx]}")
