"""GPU kernels vs the CPU oracle, stage by stage, through the C ABI.

Bit-exact: projection (visible set, compact maps, depths, tile counts,
projected rows), binning (depth order, sorted (tile, splat) list, tile
ranges), the compositing forward (image, visible marks, used range ends), the
loss (partials, gradient), and every optimizer given identical gradients.
Within 1e-4 (mixed abs/rel): the rasterizer backward, whose atomics sum in a
different order.
"""
import numpy as np
import pytest
import torch

import oracle
from vauss_b200 import ops, scenes
from tests.helpers import assert_bits_equal, assert_mixed_close, medium_scene, tiny_scene

pytestmark = pytest.mark.gpu


def _t(a, dev, dtype=None):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev) if dtype is None else \
        torch.from_numpy(np.ascontiguousarray(a)).to(dev, dtype)


def _np(t):
    return t.detach().cpu().numpy()


def _render_both(sp, cam, dev, mip=True, bg=(0.0, 0.0, 0.0), sh_half=False):
    deg = sp.sh_degree
    cfg_o = oracle.make_cfg(deg, mip=mip, sh_half=sh_half, bg=bg)
    sh_host = sp.sh.astype(np.float16).view(np.uint16) if sh_half else sp.sh
    ref = oracle.render_forward(cam, cfg_o, scenes.SplatSet(sp.transforms, sh_host, sp.raw_opac), bg=bg)
    cfg = ops.render_cfg(deg, mip=mip, sh_half=sh_half, background=bg)
    sh_dev = _t(sp.sh.astype(np.float16), dev) if sh_half else _t(sp.sh, dev)
    out = ops.render(cam, cfg, _t(sp.transforms, dev), sh_dev, _t(sp.raw_opac, dev))
    torch.cuda.synchronize()
    return ref, out, cfg, cfg_o


CASES = [("tiny", True), ("medium", True), ("medium_default_mode", False)]


@pytest.fixture(scope="module", params=CASES, ids=[c[0] for c in CASES])
def rendered(request, cuda):
    name, mip = request.param
    if name == "tiny":
        sp, _, cams = tiny_scene()
        cam = cams[3]
    else:
        sp, cams = medium_scene()
        cam = cams[0] if mip else cams[1]
    ref, out, cfg, cfg_o = _render_both(sp, cam, cuda, mip=mip, bg=(0.1, 0.2, 0.3))
    return dict(sp=sp, cam=cam, ref=ref, out=out, cfg=cfg, cfg_o=cfg_o, dev=cuda)


def test_shared_math_bit_identical(cuda):
    x = np.concatenate([np.linspace(-87.5, 88.8, 200_001, dtype=np.float32),
                        np.float32([0.0, -0.0, 1e-30, -1e-30, 88.72283, -87.0, np.inf, -np.inf, np.nan])])
    assert_bits_equal(_np(ops.math_probe("exp", _t(x, cuda))), oracle.expf(x), "vs_expf")
    y = np.concatenate([np.exp(np.linspace(-100, 85, 200_001)).astype(np.float32),
                        np.float32([1e-45, 1e-40, 1.0, 0.0, np.inf, np.nan, -1.0])])
    assert_bits_equal(_np(ops.math_probe("log", _t(y, cuda))), oracle.logf(y), "vs_logf")


def test_projection_bit_exact(rendered):
    ref, out = rendered["ref"], rendered["out"]
    p = ref["proj"]
    f = out.frame
    assert f.num_visible == p["num_visible"]
    assert f.num_intersections == p["num_isect"]
    assert_bits_equal(_np(f.field("compact_from_global")).view(np.uint32), p["compact_from_global"], "compact_from_global")
    assert_bits_equal(_np(f.field("global_from_compact")).view(np.uint32), p["global_from_compact"], "global_from_compact")
    assert_bits_equal(_np(f.field("depths")), p["depths"], "depths")
    assert_bits_equal(_np(f.field("tile_counts")).view(np.uint32), p["tile_counts_compact"], "tile_counts")
    proj = _np(f.field("projected")).reshape(-1, 12)
    assert_bits_equal(proj[:, :9], p["projected"], "projected rows")
    assert_bits_equal(proj[:, 9].view(np.uint32), p["global_from_compact"], "projected gid lane")
    assert_bits_equal(_np(f.field("opacities")), p["opacities"], "opacities")
    assert_bits_equal(_np(f.field("max_radius")), p["max_radius"], "max_radius")


def test_binning_bit_exact(rendered):
    ref, out = rendered["ref"], rendered["out"]
    b = ref["binning"]
    f = out.frame
    assert_bits_equal(_np(f.field("depth_order")).view(np.uint32), b["depth_order"], "depth_order")
    assert_bits_equal(_np(f.field("isect_tile")).view(np.uint32), b["tile_ids"], "sorted tile ids")
    assert_bits_equal(_np(f.field("isect_compact")).view(np.uint32), b["isect_compact"], "sorted splat ids")
    assert_bits_equal(_np(f.field("tile_ranges")).view(np.uint32).reshape(-1, 2), ref["tile_offsets_pre"],
                      "tile ranges")
    # keys really are sorted by (tile, depth)
    tiles = b["tile_ids"].astype(np.uint64)
    depth_bits = ref["proj"]["depths"].view(np.uint32)[b["isect_compact"]].astype(np.uint64)
    keys = (tiles << np.uint64(32)) | depth_bits
    assert np.all(keys[1:] >= keys[:-1])


def test_raster_forward_bit_exact(rendered):
    ref, out = rendered["ref"], rendered["out"]
    assert_bits_equal(_np(out.out_img), ref["out_img"], "out_img")
    assert_bits_equal(_np(out.visible), ref["visible"], "visible")
    assert_bits_equal(_np(out.frame.field("tile_used_end")).view(np.uint32), ref["tile_offsets"][:, 1],
                      "used range ends")


def test_loss_bit_exact(rendered):
    ref, dev = rendered["ref"], rendered["dev"]
    img = ref["out_img"]
    h, w = img.shape[:2]
    rng = np.random.default_rng(5)
    gt = scenes.pack_rgba8(np.clip(img[..., :3] + 0.1 * rng.standard_normal((h, w, 3)), 0, 1))
    lo = oracle.loss_fwd(img, gt, 0.8, -0.2)
    dl = oracle.loss_bwd(img, gt, lo["coeffs"], 0.8, -0.2)
    res = ops.image_loss(_t(img, dev), _t(gt.view(np.int32), dev), 0.8, -0.2)
    torch.cuda.synchronize()
    assert_bits_equal(_np(res.partials), lo["partials"], "loss partials")
    assert_bits_equal(_np(res.dl_dpred), dl, "dL/dpred")
    assert abs(float(res.loss.item()) - lo["loss"]) <= 1e-5 * max(1.0, abs(lo["loss"]))


def test_raster_backward_close(rendered):
    ref, out, dev, cam = rendered["ref"], rendered["out"], rendered["dev"], rendered["cam"]
    rng = np.random.default_rng(11)
    v_out = (1e-3 * rng.standard_normal(ref["out_img"].shape)).astype(np.float32)
    want = oracle.raster_bwd(cam, (0.1, 0.2, 0.3), ref["proj"], ref["binning_after"], ref["out_img"], v_out)
    got = ops.rasterize_bwd(out.frame, _t(ref["out_img"], dev), _t(v_out, dev))
    torch.cuda.synchronize()
    got = _np(got)
    for lane, name in enumerate(["x", "y", "c00", "c01", "c11", "r", "g", "b", "alpha", "refine"]):
        assert_mixed_close(got[:, lane], want[:, lane], what=f"v_combined[{name}]")


def _lr_scale():
    return np.float32([1.6e-4, 1.6e-4, 1.6e-4, 2e-3, 2e-3, 2e-3, 2e-3, 5e-3, 5e-3, 5e-3])


def test_project_update_bit_exact(rendered):
    """Reference-mode fused VJP + packed Adam, given the oracle's raster gradients."""
    sp, ref, out, dev, cam = rendered["sp"], rendered["ref"], rendered["out"], rendered["dev"], rendered["cam"]
    rng = np.random.default_rng(3)
    v = ref["proj"]["num_visible"]
    vc = (1e-3 * rng.standard_normal((v, 10))).astype(np.float32)
    vc[rng.random(v) < 0.1] = 0.0  # some visible splats without gradient
    n = sp.n
    w_t = rng.integers(0, 2**32, size=(n, 10), dtype=np.uint64).astype(np.uint32) & np.uint32(0x3fff7fff)
    w_o = rng.integers(0, 2**32, size=n, dtype=np.uint64).astype(np.uint32) & np.uint32(0x3fff7fff)
    b1, b2, inv1, inv2 = ops.adam_coefficients(7)
    want = oracle.project_update(cam, rendered["cfg_o"], sp.transforms, sp.sh, sp.raw_opac,
                                 ref["proj"]["compact_from_global"], vc, w_t, _lr_scale(), w_o, b1, b2, inv1, inv2,
                                 1e-15, 0.012, 0.005 / n, 7)
    t, o = _t(sp.transforms, dev), _t(sp.raw_opac, dev)
    wt, wo = _t(w_t.view(np.int32), dev), _t(w_o.view(np.int32), dev)
    color_dir = torch.full((n + 1, 6), -7.0, device=dev)
    refine, gsq = torch.empty(n, device=dev), torch.empty(n, device=dev)
    var0 = rng.random(n).astype(np.float32) * 1e-6
    var = _t(var0, dev)
    adam = ops.N.AdamCfg(b1, b2, inv1, inv2, 1e-15, 0.012, 0.005 / n, 7)
    ops.project_update(out.frame, rendered["cfg"], t, _t(sp.sh, dev), o, _t(vc, dev), wt, _lr_scale(), wo, adam,
                       color_dir, refine, gsq, variance=var)
    torch.cuda.synchronize()
    assert_bits_equal(_np(t), want["transforms"], "transforms")
    assert_bits_equal(_np(o), want["raw_opac"], "raw_opac")
    assert_bits_equal(_np(wt).view(np.uint32), want["w_t"], "w_t")
    assert_bits_equal(_np(wo).view(np.uint32), want["w_o"], "w_o")
    assert_bits_equal(_np(color_dir)[: v + 1], want["color_dir"][: v + 1], "color_dir")
    assert_bits_equal(_np(refine), want["refine"], "v_refine")
    assert_bits_equal(_np(gsq), want["grad_sq"], "grad_sq")
    vis = ref["proj"]["compact_from_global"] > 0
    b2f = np.float32(b2)
    want_var = np.where(vis, var0 * b2f + want["grad_sq"] * np.float32(np.float32(1) - b2f), var0).astype(np.float32)
    assert_bits_equal(_np(var), want_var, "reduced SH variance")


def test_sh_step_bit_exact(cuda):
    rng = np.random.default_rng(21)
    n, rw = 3001, 48
    params = (0.1 * rng.standard_normal((n, 16, 3))).astype(np.float16)
    rows = np.zeros(n, np.uint32)
    vis = rng.random(n) < 0.6
    rows[vis] = np.arange(1, vis.sum() + 1, dtype=np.uint32)
    cd = np.zeros((n + 1, 6), np.float32)
    cd[1:, :3] = 1e-3 * rng.standard_normal((n, 3))
    d = rng.standard_normal((n, 3))
    cd[1:, 3:] = (d / np.linalg.norm(d, axis=1, keepdims=True)).astype(np.float32)
    blocks = (n * rw + 127) // 128
    codes = rng.integers(0, 2**32, size=blocks * 32, dtype=np.uint64).astype(np.uint32)
    scales = (rng.random(blocks) * 1e-4).astype(np.float32)
    var = (rng.random(n) * 1e-6).astype(np.float32)
    lrs = np.repeat(np.float32([1.0] + [0.1] * 15), 3)
    args = (0.9, np.float32(1) - np.float32(0.9), 1.2, 1.01, 1e-15, 2e-3, 5)
    wp, wc, ws = oracle.sh_step_ref(params.view(np.uint16), cd, rows, codes, scales, var, lrs, *args)
    p = _t(params, cuda)
    c, s = _t(codes.view(np.int32), cuda), _t(scales, cuda)
    ops.sh_step(p, _t(cd, cuda), _t(rows.view(np.int32), cuda), c, s, _t(var, cuda), lrs, *args)
    torch.cuda.synchronize()
    assert_bits_equal(_np(p).view(np.uint16), wp, "f16 SH params")
    assert_bits_equal(_np(c).view(np.uint32), wc, "moment codes")
    assert_bits_equal(_np(s), ws, "moment scales")


def _q8_host(count, rng):
    blocks = (count + 255) // 256
    return dict(mc=rng.integers(60, 196, size=count).astype(np.uint8), vc=rng.integers(0, 255, size=count).astype(np.uint8),
                ms=(rng.random(blocks) * 1e-4).astype(np.float32), vs=(rng.random(blocks) * 1e-4).astype(np.float32))


def _q8_dev(h, dev):
    m = ops.Q8Moments.__new__(ops.Q8Moments)
    m.m_codes, m.v_codes = _t(h["mc"], dev), _t(h["vc"], dev)
    m.m_scales, m.v_scales = _t(h["ms"], dev), _t(h["vs"], dev)
    return m


def _oracle_q8_step(sp, cam, cfg_o, proj, vc, visible, mom, time, lr_t, lr_dc, lr_rest, lr_o, opac_reg, noise):
    """Oracle composite of the fused single-view Q8 step."""
    n = sp.n
    b1, b2, inv1, inv2 = ops.adam_coefficients(time)
    grads, refine = oracle.vjp_dense(cam, cfg_o, sp.transforms, sp.sh, sp.raw_opac, proj["compact_from_global"], vc)
    width = grads.shape[1]
    if opac_reg:
        o = (np.float32(1) / (np.float32(1) + oracle.expf(-sp.raw_opac))).astype(np.float32)
        reg = (np.float32(opac_reg) * o * (np.float32(1) - o)).astype(np.float32)
        grads[:, -1] = (grads[:, -1] + reg).astype(np.float32)
    out = {}
    res_t = oracle.adam_q8(sp.transforms, grads, width, 0, 10, mom["t"]["mc"], mom["t"]["vc"], mom["t"]["ms"],
                           mom["t"]["vs"], lr_t, 1.0, b1, b2, inv1, inv2, 1e-15, time ^ (10 << 24))
    wsh = sp.sh.shape[1] * 3
    lr_sh = np.float32([lr_dc] * 3 + [lr_rest] * (wsh - 3))
    res_sh = oracle.adam_q8(sp.sh.reshape(n, -1), grads, width, 10, wsh, mom["sh"]["mc"], mom["sh"]["vc"],
                            mom["sh"]["ms"], mom["sh"]["vs"], lr_sh, 1.0, b1, b2, inv1, inv2, 1e-15, time ^ (48 << 24))
    res_o = oracle.adam_q8(sp.raw_opac, grads, width, width - 1, 1, mom["o"]["mc"], mom["o"]["vc"], mom["o"]["ms"],
                           mom["o"]["vs"], np.float32([lr_o]), 1.0, b1, b2, inv1, inv2, 1e-15, time ^ (1 << 24))
    tr = res_t[0].reshape(n, 10)
    if noise is not None:
        scale, limit, seed = noise
        tr = oracle.noise_means(tr, proj["opacities"], visible, scale, limit, seed)
    out.update(transforms=tr, t=res_t, sh=res_sh, o=res_o, refine=refine)
    return out


def test_q8_fused_step_bit_exact(rendered):
    sp, ref, out, dev, cam = rendered["sp"], rendered["ref"], rendered["out"], rendered["dev"], rendered["cam"]
    rng = np.random.default_rng(9)
    n = sp.n
    v = ref["proj"]["num_visible"]
    vc = (1e-3 * rng.standard_normal((v, 10))).astype(np.float32)
    vc[rng.random(v) < 0.1] = 0.0
    mom = dict(t=_q8_host(n * 10, rng), sh=_q8_host(sp.sh.size, rng), o=_q8_host(n, rng))
    time = 5
    lr_t = np.float32([1e-3, 1e-3, 1e-3, 2e-3, 2e-3, 2e-3, 2e-3, 5e-3, 5e-3, 5e-3])
    visible = ref["visible"]
    noise = (1e-3, 0.01, 1234)
    want = _oracle_q8_step(sp, cam, rendered["cfg_o"], ref["proj"], vc, visible, mom, time, lr_t, 2.5e-3, 2.5e-4,
                           5e-2, 1e-6, noise)
    t, sh, o = _t(sp.transforms, dev), _t(sp.sh, dev), _t(sp.raw_opac, dev)
    mt, msh, mo = _q8_dev(mom["t"], dev), _q8_dev(mom["sh"], dev), _q8_dev(mom["o"], dev)
    q8 = ops.q8_cfg(time, lr_t, 2.5e-3, 2.5e-4, 5e-2, opac_reg=1e-6, noise_scale=noise[0], noise_limit=noise[1],
                    noise_seed=noise[2])
    rn, vcount, ms_ = (torch.zeros(n, device=dev) for _ in range(3))
    ops.step_q8(out.frame, rendered["cfg"], t, sh, o, _t(vc, dev), mt, msh, mo, q8, visible=_t(visible, dev),
                refine_norm=rn, vis_count=vcount, max_screen=ms_)
    torch.cuda.synchronize()
    assert_bits_equal(_np(t), want["transforms"], "transforms")
    assert_bits_equal(_np(sh).reshape(n, -1), want["sh"][0], "sh")
    assert_bits_equal(_np(o), want["o"][0], "raw_opac")
    for name, dm, res in (("t", mt, want["t"]), ("sh", msh, want["sh"]), ("o", mo, want["o"])):
        assert_bits_equal(_np(dm.m_codes), res[1], f"{name} m codes")
        assert_bits_equal(_np(dm.v_codes), res[2], f"{name} v codes")
        assert_bits_equal(_np(dm.m_scales), res[3], f"{name} m scales")
        assert_bits_equal(_np(dm.v_scales), res[4], f"{name} v scales")
    assert_bits_equal(_np(rn), want["refine"], "refine stats")
    assert_bits_equal(_np(vcount), visible, "visibility count")
    assert_bits_equal(_np(ms_), ref["proj"]["max_radius"], "max screen radius")


@pytest.mark.parametrize("deg", [1, 2])
def test_q8_fused_step_other_sh_degrees(cuda, deg):
    sp, cams = medium_scene(seed=40 + deg, n=9_000, sh_degree=deg)
    cam = cams[0]
    ref, out, cfg, cfg_o = _render_both(sp, cam, cuda)
    rng = np.random.default_rng(deg)
    n, v = sp.n, ref["proj"]["num_visible"]
    vc = (1e-3 * rng.standard_normal((v, 10))).astype(np.float32)
    mom = dict(t=_q8_host(n * 10, rng), sh=_q8_host(sp.sh.size, rng), o=_q8_host(n, rng))
    lr_t = np.float32([1e-3] * 3 + [2e-3] * 4 + [5e-3] * 3)
    want = _oracle_q8_step(sp, cam, cfg_o, ref["proj"], vc, ref["visible"], mom, 2, lr_t, 2.5e-3, 2.5e-4, 5e-2, 0.0,
                           None)
    t, sh, o = _t(sp.transforms, cuda), _t(sp.sh, cuda), _t(sp.raw_opac, cuda)
    mt, msh, mo = _q8_dev(mom["t"], cuda), _q8_dev(mom["sh"], cuda), _q8_dev(mom["o"], cuda)
    ops.step_q8(out.frame, cfg, t, sh, o, _t(vc, cuda), mt, msh, mo, ops.q8_cfg(2, lr_t, 2.5e-3, 2.5e-4, 5e-2))
    torch.cuda.synchronize()
    assert_bits_equal(_np(t), want["transforms"], "transforms")
    assert_bits_equal(_np(sh).reshape(n, -1), want["sh"][0], "sh")
    assert_bits_equal(_np(msh.m_codes), want["sh"][1], "sh m codes")
    assert_bits_equal(_np(msh.v_scales), want["sh"][4], "sh v scales")
    assert_bits_equal(_np(o), want["o"][0], "raw_opac")


def test_dense_vjp_and_q8_dense_bit_exact(rendered):
    sp, ref, out, dev, cam = rendered["sp"], rendered["ref"], rendered["out"], rendered["dev"], rendered["cam"]
    rng = np.random.default_rng(4)
    n = sp.n
    v = ref["proj"]["num_visible"]
    vc = (1e-3 * rng.standard_normal((v, 10))).astype(np.float32)
    base = (1e-4 * rng.standard_normal((n, 10 + sp.sh.shape[1] * 3 + 1))).astype(np.float32)
    want_g, want_r = oracle.vjp_dense(cam, rendered["cfg_o"], sp.transforms, sp.sh, sp.raw_opac,
                                      ref["proj"]["compact_from_global"], vc, grads=base.copy(),
                                      refine=np.zeros(n, np.float32))
    g = _t(base, dev)
    r = torch.zeros(n, device=dev)
    ops.vjp_dense(out.frame, rendered["cfg"], _t(sp.transforms, dev), _t(sp.sh, dev), _t(sp.raw_opac, dev),
                  _t(vc, dev), g, r)
    torch.cuda.synchronize()
    assert_bits_equal(_np(g), want_g, "dense grads")
    assert_bits_equal(_np(r), want_r, "refine")
    # Adam from the dense gradient
    mom = dict(t=_q8_host(n * 10, rng), sh=_q8_host(sp.sh.size, rng), o=_q8_host(n, rng))
    time = 3
    b1, b2, inv1, inv2 = ops.adam_coefficients(time)
    width = want_g.shape[1]
    lr_t = np.float32([1e-3] * 3 + [2e-3] * 4 + [5e-3] * 3)
    wsh = sp.sh.shape[1] * 3
    lr_sh = np.float32([2.5e-3] * 3 + [2.5e-4] * (wsh - 3))
    res_t = oracle.adam_q8(sp.transforms, want_g, width, 0, 10, mom["t"]["mc"], mom["t"]["vc"], mom["t"]["ms"],
                           mom["t"]["vs"], lr_t, 1.0, b1, b2, inv1, inv2, 1e-15, time ^ (10 << 24))
    res_sh = oracle.adam_q8(sp.sh.reshape(n, -1), want_g, width, 10, wsh, mom["sh"]["mc"], mom["sh"]["vc"],
                            mom["sh"]["ms"], mom["sh"]["vs"], lr_sh, 1.0, b1, b2, inv1, inv2, 1e-15, time ^ (48 << 24))
    res_o = oracle.adam_q8(sp.raw_opac, want_g, width, width - 1, 1, mom["o"]["mc"], mom["o"]["vc"], mom["o"]["ms"],
                           mom["o"]["vs"], np.float32([5e-2]), 1.0, b1, b2, inv1, inv2, 1e-15, time ^ (1 << 24))
    t, sh, o = _t(sp.transforms, dev), _t(sp.sh, dev), _t(sp.raw_opac, dev)
    mt, msh, mo = _q8_dev(mom["t"], dev), _q8_dev(mom["sh"], dev), _q8_dev(mom["o"], dev)
    q8 = ops.q8_cfg(time, lr_t, 2.5e-3, 2.5e-4, 5e-2)
    ops.adam_q8_dense(sp.sh_degree, t, sh, o, g, mt, msh, mo, q8)
    torch.cuda.synchronize()
    assert_bits_equal(_np(t).reshape(-1), res_t[0].reshape(-1), "transforms")
    assert_bits_equal(_np(sh).reshape(n, -1), res_sh[0], "sh")
    assert_bits_equal(_np(o), res_o[0], "raw_opac")
    assert_bits_equal(_np(mt.m_codes), res_t[1], "t m codes")
    assert_bits_equal(_np(msh.v_codes), res_sh[2], "sh v codes")
    assert_bits_equal(_np(mo.v_scales), res_o[4], "o v scales")


def test_housekeeping_bit_exact(cuda):
    rng = np.random.default_rng(13)
    n = 10_000
    t = rng.standard_normal((n, 10)).astype(np.float32)
    opac = rng.random(n).astype(np.float32) * 0.2
    vis = (rng.random(n) < 0.5).astype(np.float32)
    want = oracle.noise_means(t, opac, vis, 0.01, 0.05, 77)
    tt = _t(t, cuda)
    ops.noise_means(tt, _t(opac, cuda), _t(vis, cuda), 0.01, 0.05, 77)
    torch.cuda.synchronize()
    assert_bits_equal(_np(tt), want, "noise_means")
    assert not np.array_equal(want, t)
    a, b, c = (rng.random(n).astype(np.float32) for _ in range(3))
    w, r = rng.random(n).astype(np.float32), rng.random(n).astype(np.float32)
    wn, wv, ws = oracle.gather_stats(a, b, c, w, vis, r)
    ta, tb, tc = _t(a, cuda), _t(b, cuda), _t(c, cuda)
    ops.gather_stats(ta, tb, tc, _t(w, cuda), _t(vis, cuda), _t(r, cuda))
    torch.cuda.synchronize()
    assert_bits_equal(_np(ta), wn, "refine max")
    assert_bits_equal(_np(tb), wv, "visible sum")
    assert_bits_equal(_np(tc), ws, "radius max")


def test_f16_sh_render_bit_exact(cuda):
    sp, cams = medium_scene(seed=8, n=20_000)
    ref, out, _, _ = _render_both(sp, cams[0], cuda, sh_half=True)
    assert_bits_equal(_np(out.out_img), ref["out_img"], "out_img (f16 SH)")
