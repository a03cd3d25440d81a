"""The dataset feed's host side: packing (the oracle against the reference's
own unit tests in crates/splat-train-dataset/src/scene.rs:202-240) and the
visiting order (vs_feed_order, host-only)."""
import numpy as np
import pytest

import oracle
from vauss_b200 import dataset


def test_pack_golden_vectors_from_reference_tests():
    # packs_rgba_samples_without_changing_channels (scene.rs:206-219)
    px = np.array([[[1, 2, 3, 4], [5, 6, 7, 8]]], np.uint8)
    out, has_alpha = oracle.pack_view(px, dataset.AlphaMode.MASKED)
    assert has_alpha and out.shape == (1, 2)
    assert out.ravel().tolist() == [0x04030201, 0x08070605]
    # fills_missing_alpha_with_opaque_for_rgb_samples (scene.rs:221-240)
    px = np.array([[[9, 10, 11], [12, 13, 14]]], np.uint8)
    out, has_alpha = oracle.pack_view(px, dataset.AlphaMode.TRANSPARENT)
    assert not has_alpha
    assert out.ravel().tolist() == [0xff0b0a09, 0xff0e0d0c]


def test_pack_premultiplies_in_byte_space_only_when_transparent():
    px = np.array([[[200, 100, 50, 128], [255, 255, 255, 0], [7, 8, 9, 255]]], np.uint8)
    masked, _ = oracle.pack_view(px, 0)
    assert masked.ravel().tolist() == [0x803264C8, 0x00FFFFFF, 0xFF090807]
    trans, _ = oracle.pack_view(px, 1)
    # (c * a + 127) / 255: 200 -> 100, 100 -> 50, 50 -> 25 at a = 128; a = 0 clears
    assert trans.ravel().tolist() == [0x80193264, 0x00000000, 0xFF090807]


def test_pack_widens_luma():
    l8 = np.array([[3, 250]], np.uint8)
    out, has_alpha = oracle.pack_view(l8, 1)
    assert not has_alpha and out.ravel().tolist() == [0xFF030303, 0xFFFAFAFA]
    la = np.array([[[100, 51]]], np.uint8)
    out, has_alpha = oracle.pack_view(la, 1)
    assert has_alpha and out.ravel().tolist() == [(51 << 24) | 0x141414]  # 100 * 51 -> 20


@pytest.mark.parametrize("n", [1, 2, 7, 64])
def test_visiting_order_is_epochs_of_permutations(native_lib, n):
    order = dataset.visiting_order(1234, n, 5 * n)
    for e in range(5):
        assert sorted(order[e * n:(e + 1) * n]) == list(range(n))
    assert order == dataset.visiting_order(1234, n, 5 * n)
    if n >= 7:
        assert order != dataset.visiting_order(1235, n, 5 * n)
        assert order[:n] != order[n:2 * n]


def test_shard_is_round_robin():
    sc = dataset.Scene([dataset.SceneView(np.zeros((2, 2, 3), np.uint8), None) for _ in range(10)])
    parts = [dataset.shard(sc, r, 4) for r in range(4)]
    assert [len(p.views) for p in parts] == [3, 3, 2, 2]
    assert parts[1].views[0] is sc.views[1] and parts[1].views[1] is sc.views[5]
