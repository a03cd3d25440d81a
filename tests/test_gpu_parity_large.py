"""GPU vs the CPU oracle at the size of BASELINE.json configs[1]: 1M SH-3
splats, one 1920x1080 view at distance 6 (fx = fy = 1600), Mip mode, an
upstream image gradient N(0, 1e-3) per pixel and channel.

At this size the projection has ~0.66M visible splats and the binning ~3.6M
intersections, so the multi-chunk scans, multi-batch tiles and more than
65k-block grids all run.  Projection and binning are compared bit for bit
(compact maps, depths, tile counts, projected rows, sorted (tile, splat)
lists, tile ranges before and after the forward); the rendered image, the
visible marks and the rasterizer backward's v_combined are compared within
the tests' tolerance (tests/helpers.py)."""
import os

import numpy as np
import pytest
import torch

import oracle
from vauss_b200 import ops, scenes
from tests.helpers import assert_bits_equal, assert_mixed_close

pytestmark = pytest.mark.gpu


def _np(t):
    return t.detach().cpu().numpy()


@pytest.fixture(scope="module")
def config1(cuda):
    oracle.set_num_threads(os.cpu_count() or 1)
    sp, cam = scenes.config_microbench()
    cfg_o = oracle.make_cfg(3, mip=True)
    ref = oracle.render_forward(cam, cfg_o, sp)
    v_out = (np.random.default_rng(11).standard_normal((cam.height, cam.width, 4)) * 1e-3).astype(np.float32)
    vc_ref = oracle.raster_bwd(cam, (0.0, 0.0, 0.0), ref["proj"], ref["binning_after"], ref["out_img"], v_out)
    cfg = ops.render_cfg(3, mip=True)
    t, sh, o = (torch.from_numpy(x).to(cuda) for x in (sp.transforms, sp.sh, sp.raw_opac))
    out = ops.render(cam, cfg, t, sh, o)
    vc = ops.rasterize_bwd(out.frame, out.out_img, torch.from_numpy(v_out).to(cuda))
    torch.cuda.synchronize()
    return dict(ref=ref, vc_ref=vc_ref, out=out, vc=_np(vc), cam=cam)


def test_config1_sizes(config1):
    f, p = config1["out"].frame, config1["ref"]["proj"]
    assert f.num_visible == p["num_visible"] > 500_000
    assert f.num_intersections == p["num_isect"] > 3_000_000


def test_config1_projection_bit_exact(config1):
    f, p = config1["out"].frame, config1["ref"]["proj"]
    assert_bits_equal(_np(f.field("compact_from_global")).view(np.uint32), p["compact_from_global"],
                      "compact_from_global")
    assert_bits_equal(_np(f.field("global_from_compact")).view(np.uint32), p["global_from_compact"],
                      "global_from_compact")
    assert_bits_equal(_np(f.field("depths")), p["depths"], "depths")
    assert_bits_equal(_np(f.field("tile_counts")).view(np.uint32), p["tile_counts_compact"], "tile counts")
    proj = _np(f.field("projected")).reshape(-1, 12)
    assert_bits_equal(proj[:, :9], p["projected"], "projected rows")


def test_config1_binning_bit_exact(config1):
    ref, f = config1["ref"], config1["out"].frame
    b = ref["binning"]
    assert_bits_equal(_np(f.field("depth_order")).view(np.uint32), b["depth_order"], "depth order")
    assert_bits_equal(_np(f.field("isect_tile")).view(np.uint32), b["tile_ids"], "sorted tile ids")
    assert_bits_equal(_np(f.field("isect_compact")).view(np.uint32), b["isect_compact"], "sorted splat ids")
    assert_bits_equal(_np(f.field("tile_ranges")).view(np.uint32).reshape(-1, 2), ref["tile_offsets_pre"],
                      "tile ranges")
    tiles = b["tile_ids"].astype(np.uint64)
    depth_bits = ref["proj"]["depths"].view(np.uint32)[b["isect_compact"]].astype(np.uint64)
    keys = (tiles << np.uint64(32)) | depth_bits
    assert np.all(keys[1:] >= keys[:-1])


def test_config1_forward(config1):
    ref, out = config1["ref"], config1["out"]
    assert_mixed_close(_np(out.out_img), ref["out_img"], what="image")
    assert np.array_equal(_np(out.visible), ref["visible"]), "visible marks"
    assert_bits_equal(_np(out.frame.field("tile_used_end")).view(np.uint32), ref["tile_offsets"][:, 1],
                      "used range ends")


def test_config1_backward(config1):
    assert_mixed_close(config1["vc"], config1["vc_ref"], what="v_combined")
