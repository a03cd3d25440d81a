"""The inference render (vs_render_image, the reference's RasterPass::Forward):
packed RGBA8 pixels equal to the oracle's float render packed the reference's
way (kernels/rasterize.rs:401-409: clamp(255 c, 0, 255) converted toward
zero, r in the low byte), bit for bit, in both render modes and with f16 SH."""
import numpy as np
import pytest
import torch

import oracle
from vauss_b200 import ops, scenes
from tests.helpers import assert_bits_equal, medium_scene

pytestmark = pytest.mark.gpu


def pack_reference(img):
    """[H, W, 4] f32 -> [H, W] u32, in float32 arithmetic like the kernel."""
    q = np.clip(img.astype(np.float32) * np.float32(255.0), np.float32(0.0), np.float32(255.0)).astype(np.uint32)
    return q[..., 0] | (q[..., 1] << 8) | (q[..., 2] << 16) | (q[..., 3] << 24)


@pytest.mark.parametrize("mip,half", [(True, False), (False, False), (True, True)])
def test_inference_render_matches_oracle(cuda, mip, half):
    sp, cams = medium_scene(seed=61, n=30_000, sh_degree=3)
    bg = (0.2, 0.4, 0.6)
    # the oracle reads f16 coefficients as their raw 16-bit words
    sp_o = scenes.SplatSet(sp.transforms, sp.sh.astype(np.float16).view(np.uint16), sp.raw_opac) if half else sp
    for cam in cams:
        want = pack_reference(oracle.render_forward(cam, oracle.make_cfg(3, mip=mip, bg=bg, sh_half=half), sp_o,
                                                    bg=bg)["out_img"])
        sh = torch.from_numpy(sp.sh).to(cuda)
        if half:
            sh = sh.half()
        cfg = ops.render_cfg(3, mip=mip, sh_half=half, background=bg)
        t, o = torch.from_numpy(sp.transforms).to(cuda), torch.from_numpy(sp.raw_opac).to(cuda)
        got = ops.render_image(cam, cfg, t, sh, o)
        train = ops.render(cam, cfg, t, sh, o).out_img
        torch.cuda.synchronize()
        got = got.cpu().numpy().view(np.uint32)
        assert_bits_equal(got, want, "packed image vs oracle")
        assert_bits_equal(got, pack_reference(train.cpu().numpy()), "packed image vs training render")
