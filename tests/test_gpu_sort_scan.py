"""The GPU radix sort and scan against the reference's own known-answer tests
(crates/splat-train-sort/src/lib.rs:219-404, crates/splat-train-scan/src/
lib.rs:120-254), restated."""
import numpy as np
import pytest
import torch

import oracle
from vauss_b200 import ops

pytestmark = pytest.mark.gpu


def _sort(keys: np.ndarray, vals: np.ndarray, bits: int = 32):
    k = torch.from_numpy(keys.view(np.int32).copy()).cuda()
    v = torch.from_numpy(vals.view(np.int32).copy()).cuda()
    ops.radix_sort_pairs(k, v, bits)
    torch.cuda.synchronize()
    return k.cpu().numpy().view(np.uint32), v.cpu().numpy().view(np.uint32)


def test_sort_fixed_patterns(cuda):
    for i in range(128):
        keys = np.array([5 + i * 4, i, 6, 123, 74657, 123, 999, 2 ** 24 + 123, 6, 7, 8, 0, i * 2, 16 + i, 128 * i],
                        dtype=np.uint32)
        vals = keys * 2 + 5
        order = np.argsort(keys, kind="stable")
        k, v = _sort(keys, vals)
        assert np.array_equal(k, keys[order]) and np.array_equal(v, vals[order])


def test_sort_gaussian_like_keys(cuda):
    rng = np.random.default_rng(0)
    keys = []
    for i in range(10000):
        start = rng.integers(i, i + 150)
        end = rng.integers(start, start + 250)
        span = np.arange(start, end)
        keys.append(span[rng.random(span.size) < 0.5])
    keys = np.concatenate(keys).astype(np.uint32)
    vals = keys * 2 + 5
    order = np.argsort(keys, kind="stable")
    k, v = _sort(keys, vals)
    assert np.array_equal(k, keys[order]) and np.array_equal(v, vals[order])


def test_sort_large_is_sorted_and_stable(cuda):
    rng = np.random.default_rng(1)
    n = 30_000_000
    keys = rng.integers(0, 1_000_000, size=n, dtype=np.uint32)
    vals = np.arange(n, dtype=np.uint32)
    k, v = _sort(keys, vals)
    assert np.all(k[1:] >= k[:-1])
    same = k[1:] == k[:-1]
    assert np.all(v[1:][same] > v[:-1][same]), "not stable"
    assert np.array_equal(keys[v], k)


def test_sort_above_67m_keys_kat(cuda):
    n = 70_000_000
    keys = oracle.splitmix_shuffle(n, 0xD15EA5E)
    vals = np.arange(n, dtype=np.uint32)
    expected = np.empty(n, np.uint32)
    expected[keys] = vals
    k, v = _sort(keys, vals)
    assert np.array_equal(k, np.arange(n, dtype=np.uint32))
    assert np.array_equal(v, expected)


@pytest.mark.parametrize("bits", [1, 5, 8, 9, 13, 16, 17, 18, 24, 26, 27, 28])
def test_sort_partial_bit_ranges(cuda, bits):
    rng = np.random.default_rng(bits)
    keys = rng.integers(0, 2 ** bits, size=200_001, dtype=np.uint32)
    vals = rng.integers(0, 2 ** 32, size=keys.size, dtype=np.uint64).astype(np.uint32)
    order = np.argsort(keys, kind="stable")
    k, v = _sort(keys, vals, bits)
    assert np.array_equal(k, keys[order]) and np.array_equal(v, vals[order])


def test_scan_known_answers(cuda):
    x = torch.ones(4, dtype=torch.int32, device="cuda")
    assert ops.scan_inclusive(x) == 4
    assert x.cpu().tolist() == [1, 2, 3, 4]
    rng = np.random.default_rng(2)
    for n in (1, 255, 256, 257, 1023, 1024, 1025, 2048, 2049, 4095, 4096, 4097, (1 << 20) + 1):
        a = rng.integers(0, 1000, size=n, dtype=np.uint32)
        t = torch.from_numpy(a.view(np.int32).copy()).cuda()
        total = ops.scan_inclusive(t)
        want = np.cumsum(a.astype(np.uint64))
        assert total == int(want[-1])
        assert np.array_equal(t.cpu().numpy().view(np.uint32), want.astype(np.uint32))


def test_scan_30m(cuda):
    n = 30_000_000
    t = torch.ones(n, dtype=torch.int32, device="cuda")
    assert ops.scan_inclusive(t) == n
    assert int(t[-1].item()) == n and int(t[n // 2].item()) == n // 2 + 1
