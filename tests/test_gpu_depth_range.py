"""Binning over depth ranges of every width, GPU against the CPU oracle.

The depth sort runs over the bits in which the visible splats' depths differ
(the keys are the depth bits less the smallest one), in ceil(bits / 9)
passes.  These scenes put the splats at chosen camera-space depths -- all one
depth (no key bits: the order is the compact order), a handful of adjacent
floats, a 3-pass range and a wide range that needs four passes -- and require
the projection, the depth order, the sorted intersection list, the tile
ranges and the image to equal the oracle's bit for bit.
"""
import numpy as np
import pytest
import torch

import oracle
from vauss_b200 import ops, scenes
from vauss_b200.camera import Camera
from tests.helpers import assert_bits_equal

pytestmark = pytest.mark.gpu

W, H, FX = 240, 176, 220.0


def _camera() -> Camera:
    # at the origin, looking along +z: a splat's depth is its z coordinate
    return Camera(R=np.eye(3, dtype=np.float32), t=np.zeros(3, np.float32), fx=FX, fy=FX, cx=0.5 * W, cy=0.5 * H,
                  width=W, height=H)


def _splats_at(z: np.ndarray, seed: int) -> scenes.SplatSet:
    """Splats inside the view at depths z, sized to cover a few pixels."""
    n = z.size
    sp = scenes.random_splats(n, seed, mean_lo=0.0, mean_hi=1.0, log_scale_mu=0.0, log_scale_sigma=0.3,
                              opac_mu=0.5, opac_sigma=1.0, sh_degree=1)
    rng = np.random.default_rng(seed + 1)
    z = z.astype(np.float32)
    sp.transforms[:, 0] = (rng.uniform(-0.5, 0.5, n) * (W / FX) * z).astype(np.float32)
    sp.transforms[:, 1] = (rng.uniform(-0.5, 0.5, n) * (H / FX) * z).astype(np.float32)
    sp.transforms[:, 2] = z
    # about 2-6 pixels across at any depth
    sp.transforms[:, 7:10] = (np.log(z * (3.0 / FX))[:, None]
                              + 0.3 * rng.standard_normal((n, 3))).astype(np.float32)
    return sp


def _depths(kind: str, n: int) -> np.ndarray:
    rng = np.random.default_rng(11)
    if kind == "one_depth":
        return np.full(n, 3.0, np.float32)
    if kind == "adjacent_floats":
        bits = np.uint32(np.float32(3.0).view(np.uint32)) + rng.integers(0, 5, n).astype(np.uint32)
        return bits.view(np.float32)
    if kind == "three_passes":
        return rng.uniform(1.5, 6.5, n).astype(np.float32)
    assert kind == "four_passes"
    return np.exp(rng.uniform(np.log(0.05), np.log(2.0e4), n)).astype(np.float32)


def _key_bits(depths: np.ndarray) -> int:
    b = depths.view(np.uint32)
    span = int(b.max()) - int(b.min())
    return span.bit_length()


@pytest.mark.parametrize("kind,want_bits", [("one_depth", (0, 0)), ("adjacent_floats", (1, 3)),
                                            ("three_passes", (19, 27)), ("four_passes", (28, 32))])
def test_binning_over_depth_ranges(cuda, kind, want_bits):
    sp = _splats_at(_depths(kind, 6000), seed=5)
    cam = _camera()
    cfg_o = oracle.make_cfg(1, mip=True, bg=(0.0, 0.0, 0.0))
    ref = oracle.render_forward(cam, cfg_o, sp, bg=(0.0, 0.0, 0.0))
    cfg = ops.render_cfg(1, mip=True, background=(0.0, 0.0, 0.0))
    dev = cuda
    out = ops.render(cam, cfg, torch.from_numpy(sp.transforms).to(dev), torch.from_numpy(sp.sh).to(dev),
                     torch.from_numpy(sp.raw_opac).to(dev))
    torch.cuda.synchronize()
    p, b, f = ref["proj"], ref["binning"], out.frame
    assert f.num_visible == p["num_visible"] and f.num_visible > 1000
    assert f.num_intersections == p["num_isect"]
    bits = _key_bits(p["depths"])
    assert want_bits[0] <= bits <= want_bits[1], f"{kind}: depth key bits {bits}"
    assert_bits_equal(f.field("depths").cpu().numpy(), p["depths"], "depths")
    assert_bits_equal(f.field("depth_order").cpu().numpy().view(np.uint32), b["depth_order"], "depth_order")
    assert_bits_equal(f.field("isect_tile").cpu().numpy().view(np.uint32), b["tile_ids"], "sorted tile ids")
    assert_bits_equal(f.field("isect_compact").cpu().numpy().view(np.uint32), b["isect_compact"], "sorted splat ids")
    assert_bits_equal(f.field("tile_ranges").cpu().numpy().view(np.uint32).reshape(-1, 2), ref["tile_offsets_pre"],
                      "tile ranges")
    assert_bits_equal(out.out_img.cpu().numpy(), ref["out_img"], "image")
