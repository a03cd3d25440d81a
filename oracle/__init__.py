"""CPU parity oracle (TEST INFRASTRUCTURE ONLY).

numpy front end of ``splat_oracle.cpp``, the host restatement of the
reference's training-step kernels.  Only ``tests/``, ``__graft_entry__.smoke``
and ``bench.py``'s CPU-baseline leg use it, always as the checker or the timed
CPU baseline, never as part of the product path.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = os.path.join(_HERE, "_build", "liboracle.so")
_lock = threading.Lock()
_lib = None

F32P = ctypes.POINTER(ctypes.c_float)
U32P = ctypes.POINTER(ctypes.c_uint32)
U16P = ctypes.POINTER(ctypes.c_uint16)
U8P = ctypes.POINTER(ctypes.c_uint8)
U64P = ctypes.POINTER(ctypes.c_uint64)
VP = ctypes.c_void_p


class RenderCfg(ctypes.Structure):
    _fields_ = [
        ("mip", ctypes.c_int32),
        ("sh_degree", ctypes.c_int32),
        ("sh_half", ctypes.c_int32),
        ("has_min_scale", ctypes.c_int32),
        ("log_scale_offset", ctypes.c_float),
        ("bg", ctypes.c_float * 3),
    ]


def make_cfg(sh_degree: int, mip: bool = True, sh_half: bool = False, bg=(0.0, 0.0, 0.0),
             log_scale_offset: float = 0.0, has_min_scale: bool = False) -> RenderCfg:
    c = RenderCfg()
    c.mip, c.sh_degree, c.sh_half, c.has_min_scale = int(mip), int(sh_degree), int(sh_half), int(has_min_scale)
    c.log_scale_offset = float(log_scale_offset)
    for i in range(3):
        c.bg[i] = float(bg[i])
    return c


def build() -> str:
    """Compile the oracle with its Makefile (g++); returns the library path."""
    with _lock:
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB) or os.path.getmtime(_LIB) < os.path.getmtime(
                os.path.join(_HERE, "splat_oracle.cpp")):
            build()
        _lib = ctypes.CDLL(_LIB)
    return _lib


def _p(a: np.ndarray, t):
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be contiguous"
    return a.ctypes.data_as(t)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def project(cam, cfg: RenderCfg, transforms, sh, raw_opac, min_scale=None):
    """K1 + K2: returns a dict of per-global and compact (global-order) arrays."""
    L = lib()
    transforms, raw_opac = _f32(transforms), _f32(raw_opac)
    n = transforms.shape[0]
    sh = np.ascontiguousarray(sh)
    ms = _f32(min_scale) if min_scale is not None else np.zeros(1, np.float32)
    c = cam.to_c()
    out = dict(
        compact_from_global=np.zeros(n, np.uint32), opacities=np.zeros(n, np.float32),
        max_radius=np.zeros(n, np.float32), tile_counts=np.zeros(n, np.uint32),
        global_from_compact=np.zeros(max(n, 1), np.uint32), depths=np.zeros(max(n, 1), np.float32),
        tile_counts_compact=np.zeros(max(n, 1), np.uint32), projected=np.zeros((max(n, 1), 9), np.float32))
    nv = ctypes.c_uint32(0)
    ni = ctypes.c_uint64(0)
    rc = L.or_project(ctypes.byref(c), ctypes.byref(cfg), ctypes.c_uint32(n), _p(transforms, F32P),
                      sh.ctypes.data_as(VP), _p(raw_opac, F32P), _p(ms, F32P),
                      _p(out["compact_from_global"], U32P), _p(out["opacities"], F32P), _p(out["max_radius"], F32P),
                      _p(out["tile_counts"], U32P), _p(out["global_from_compact"], U32P), _p(out["depths"], F32P),
                      _p(out["tile_counts_compact"], U32P), _p(out["projected"], F32P), ctypes.byref(nv),
                      ctypes.byref(ni))
    assert rc == 0
    v = nv.value
    for k in ("global_from_compact", "depths", "tile_counts_compact", "projected"):
        out[k] = out[k][:v].copy()
    out["num_visible"] = v
    out["num_isect"] = ni.value
    return out


def bin(cam, proj):
    """K3-K7: depth sort, emission, stable tile sort, tile ranges."""
    L = lib()
    v = proj["num_visible"]
    ni = int(proj["num_isect"])
    T = cam.num_tiles
    depth_order = np.zeros(max(v, 1), np.uint32)
    tile_ids = np.zeros(max(ni, 1), np.uint32)
    isect = np.zeros(max(ni, 1), np.uint32)
    offsets = np.zeros(2 * T, np.uint32)
    out_n = ctypes.c_uint64(0)
    projd = _f32(proj["projected"]) if v else np.zeros((1, 9), np.float32)
    depths = _f32(proj["depths"]) if v else np.zeros(1, np.float32)
    counts = np.ascontiguousarray(proj["tile_counts_compact"], np.uint32) if v else np.zeros(1, np.uint32)
    c = cam.to_c()
    rc = L.or_bin(ctypes.byref(c), ctypes.c_uint32(v), _p(projd, F32P), _p(depths, F32P), _p(counts, U32P),
                  ctypes.c_uint64(max(ni, 1)), _p(depth_order, U32P), _p(tile_ids, U32P), _p(isect, U32P),
                  _p(offsets, U32P), ctypes.byref(out_n))
    assert rc == 0, rc
    n = out_n.value
    return dict(depth_order=depth_order[:v].copy(), tile_ids=tile_ids[:n].copy(),
                isect_compact=isect[:n].copy(), tile_offsets=offsets.reshape(-1, 2).copy(), num_isect=n)


def raster_fwd(cam, bg, proj, binning, n_total: int):
    L = lib()
    H, W = cam.height, cam.width
    out = np.zeros((H, W, 4), np.float32)
    visible = np.zeros(n_total, np.float32)
    offsets = np.ascontiguousarray(binning["tile_offsets"].reshape(-1), np.uint32).copy()
    projd = _f32(proj["projected"]) if proj["num_visible"] else np.zeros((1, 9), np.float32)
    gfc = np.ascontiguousarray(proj["global_from_compact"], np.uint32) if proj["num_visible"] else np.zeros(1, np.uint32)
    isect = np.ascontiguousarray(binning["isect_compact"], np.uint32) if binning["num_isect"] else np.zeros(1, np.uint32)
    bgv = _f32(bg)
    c = cam.to_c()
    rc = L.or_raster_fwd(ctypes.byref(c), _p(bgv, F32P), _p(projd, F32P), _p(gfc, U32P), _p(isect, U32P),
                         _p(offsets, U32P), _p(out, F32P), _p(visible, F32P))
    assert rc == 0
    return dict(out_img=out, visible=visible, tile_offsets=offsets.reshape(-1, 2))


def loss_fwd(pred, gt_packed, l1_w: float, ssim_w: float, want_map: bool = False):
    L = lib()
    pred = _f32(pred)
    H, W = pred.shape[:2]
    assert pred.shape[2] == 4
    gt = np.ascontiguousarray(gt_packed, np.uint32)
    tiles = ((W + 15) // 16) * ((H + 15) // 16)
    partials = np.zeros((3, tiles), np.float32)
    coeffs = np.zeros((3, 3, H, W), np.float32)
    smap = np.zeros((H, W, 3), np.float32) if want_map else None
    rc = L.or_loss_fwd(ctypes.c_uint32(H), ctypes.c_uint32(W), _p(pred, F32P), _p(gt, U32P),
                       ctypes.c_float(l1_w), ctypes.c_float(ssim_w), _p(partials, F32P), _p(coeffs, F32P),
                       _p(smap, F32P) if smap is not None else None)
    assert rc == 0
    return dict(partials=partials, coeffs=coeffs, ssim_map=smap, loss=float(partials.astype(np.float64).sum()))


def loss_bwd(pred, gt_packed, coeffs, l1_w: float, ssim_w: float):
    L = lib()
    pred = _f32(pred)
    H, W = pred.shape[:2]
    gt = np.ascontiguousarray(gt_packed, np.uint32)
    coeffs = _f32(coeffs)
    out = np.zeros((H, W, 4), np.float32)
    rc = L.or_loss_bwd(ctypes.c_uint32(H), ctypes.c_uint32(W), _p(pred, F32P), _p(gt, U32P), _p(coeffs, F32P),
                       ctypes.c_float(l1_w), ctypes.c_float(ssim_w), _p(out, F32P))
    assert rc == 0
    return out


def raster_bwd(cam, bg, proj, binning_after_fwd, out_img, v_out):
    L = lib()
    v = proj["num_visible"]
    vc = np.zeros((max(v, 1), 10), np.float32)
    projd = _f32(proj["projected"]) if v else np.zeros((1, 9), np.float32)
    isect = np.ascontiguousarray(binning_after_fwd["isect_compact"], np.uint32) \
        if binning_after_fwd["num_isect"] else np.zeros(1, np.uint32)
    offsets = np.ascontiguousarray(binning_after_fwd["tile_offsets"].reshape(-1), np.uint32)
    c = cam.to_c()
    bgv = _f32(bg)
    rc = L.or_raster_bwd(ctypes.byref(c), _p(bgv, F32P), ctypes.c_uint32(v), _p(projd, F32P), _p(isect, U32P),
                         _p(offsets, U32P), _p(_f32(out_img), F32P), _p(_f32(v_out), F32P), _p(vc, F32P))
    assert rc == 0
    return vc[:v]


def project_update(cam, cfg, transforms, sh, raw_opac, compact_from_global, v_combined, w_t, lr_scale, w_o,
                   b1, b2, inv1, inv2, eps, lr_opac, opac_reg, round_seed, min_scale=None):
    """Reference-mode fused VJP + packed Adam; arrays are updated on copies."""
    L = lib()
    n = transforms.shape[0]
    t = _f32(transforms).copy()
    o = _f32(raw_opac).copy()
    wt = np.ascontiguousarray(w_t, np.uint32).copy()
    wo = np.ascontiguousarray(w_o, np.uint32).copy()
    color_dir = np.zeros((n + 1, 6), np.float32)
    refine = np.zeros(n, np.float32)
    gsq = np.zeros(n, np.float32)
    vc = _f32(v_combined) if len(v_combined) else np.zeros((1, 10), np.float32)
    ms = _f32(min_scale) if min_scale is not None else np.zeros(1, np.float32)
    sh = np.ascontiguousarray(sh)
    c = cam.to_c()
    rc = L.or_project_update(ctypes.byref(c), ctypes.byref(cfg), ctypes.c_uint32(n), _p(t, F32P),
                             sh.ctypes.data_as(VP), _p(o, F32P), _p(ms, F32P),
                             _p(np.ascontiguousarray(compact_from_global, np.uint32), U32P), _p(vc, F32P),
                             _p(wt, U32P), _p(_f32(lr_scale), F32P), _p(wo, U32P), _p(color_dir, F32P),
                             _p(refine, F32P), _p(gsq, F32P), ctypes.c_float(b1), ctypes.c_float(b2),
                             ctypes.c_float(inv1), ctypes.c_float(inv2), ctypes.c_float(eps),
                             ctypes.c_float(lr_opac), ctypes.c_float(opac_reg), ctypes.c_uint32(round_seed))
    assert rc == 0
    return dict(transforms=t, raw_opac=o, w_t=wt, w_o=wo, color_dir=color_dir, refine=refine, grad_sq=gsq)


def sh_step_ref(params_f16, color_dir, grad_rows, codes, scales, variance, lr_scale, beta, factor, inv1, inv2, eps,
                lr, round_seed):
    L = lib()
    p = np.ascontiguousarray(params_f16, np.uint16).copy()
    n = p.shape[0]
    row_width = int(np.prod(p.shape[1:]))
    cd = np.ascontiguousarray(codes, np.uint32).copy()
    sc = _f32(scales).copy()
    rc = L.or_sh_step_ref(ctypes.c_uint32(n), ctypes.c_uint32(row_width), _p(p, U16P), _p(_f32(color_dir), F32P),
                          _p(np.ascontiguousarray(grad_rows, np.uint32), U32P), _p(cd, U32P), _p(sc, F32P),
                          _p(_f32(variance), F32P), _p(_f32(lr_scale), F32P), ctypes.c_float(beta),
                          ctypes.c_float(factor), ctypes.c_float(inv1), ctypes.c_float(inv2), ctypes.c_float(eps),
                          ctypes.c_float(lr), ctypes.c_uint32(round_seed))
    assert rc == 0
    return p, cd, sc


def vjp_dense(cam, cfg, transforms, sh, raw_opac, compact_from_global, v_combined, grads=None, refine=None,
              min_scale=None):
    L = lib()
    n = transforms.shape[0]
    width = 10 + 3 * (cfg.sh_degree + 1) ** 2 + 1
    grads = np.zeros((n, width), np.float32) if grads is None else grads
    refine = np.zeros(n, np.float32) if refine is None else refine
    vc = _f32(v_combined) if len(v_combined) else np.zeros((1, 10), np.float32)
    ms = _f32(min_scale) if min_scale is not None else np.zeros(1, np.float32)
    sh = np.ascontiguousarray(sh)
    c = cam.to_c()
    rc = L.or_vjp_dense(ctypes.byref(c), ctypes.byref(cfg), ctypes.c_uint32(n), _p(_f32(transforms), F32P),
                        sh.ctypes.data_as(VP), _p(_f32(raw_opac), F32P), _p(ms, F32P),
                        _p(np.ascontiguousarray(compact_from_global, np.uint32), U32P), _p(vc, F32P),
                        _p(grads, F32P), _p(refine, F32P))
    assert rc == 0
    return grads, refine


def adam_q8(params, grads, grad_stride, grad_offset, row_width, m_codes, v_codes, m_scales, v_scales, lr_col, lr,
            b1, b2, inv1, inv2, eps, seed):
    """The benchmark's 8-bit m+v Adam on one flattened parameter tensor (copies)."""
    L = lib()
    p = _f32(params).copy()
    count = p.size
    mc = np.ascontiguousarray(m_codes, np.uint8).copy()
    vcd = np.ascontiguousarray(v_codes, np.uint8).copy()
    ms = _f32(m_scales).copy()
    vs = _f32(v_scales).copy()
    rc = L.or_adam_q8(ctypes.c_size_t(count), ctypes.c_uint32(row_width), _p(p, F32P), _p(_f32(grads), F32P),
                      ctypes.c_size_t(grad_stride), ctypes.c_size_t(grad_offset), _p(mc, U8P), _p(vcd, U8P),
                      _p(ms, F32P), _p(vs, F32P), _p(_f32(lr_col), F32P), ctypes.c_float(lr), ctypes.c_float(b1),
                      ctypes.c_float(b2), ctypes.c_float(inv1), ctypes.c_float(inv2), ctypes.c_float(eps),
                      ctypes.c_uint32(seed))
    assert rc == 0
    return p, mc, vcd, ms, vs


def gather_stats(norm, vis, screen, weight, visible, radius):
    L = lib()
    norm, vis, screen = _f32(norm).copy(), _f32(vis).copy(), _f32(screen).copy()
    rc = L.or_gather_stats(ctypes.c_uint32(norm.size), _p(norm, F32P), _p(vis, F32P), _p(screen, F32P),
                           _p(_f32(weight), F32P), _p(_f32(visible), F32P), _p(_f32(radius), F32P))
    assert rc == 0
    return norm, vis, screen


def noise_means(transforms, opacities, visible, scale, limit, seed):
    L = lib()
    t = _f32(transforms).copy()
    rc = L.or_noise_means(ctypes.c_uint32(t.shape[0]), _p(t, F32P), _p(_f32(opacities), F32P),
                          _p(_f32(visible), F32P), ctypes.c_float(scale), ctypes.c_float(limit),
                          ctypes.c_uint32(seed))
    assert rc == 0
    return t


def refine_table(transforms, sh, raw_opac, refine_weight, vis_weight, max_screen, min_opacity, max_bound, center,
                 split_at_screen_size):
    """Per-splat refine decision table [N, 8] (train.rs:1822-1883)."""
    L = lib()
    t, o = _f32(transforms), _f32(raw_opac)
    n = t.shape[0]
    shf = _f32(np.asarray(sh, np.float32).reshape(n, -1))
    table = np.zeros((max(n, 1), 8), np.float32)
    c = np.asarray(center, np.float32)
    rc = L.or_refine_table(ctypes.c_uint32(n), _p(t, F32P), _p(shf, F32P), ctypes.c_uint32(shf.shape[1]),
                           _p(o, F32P), _p(_f32(refine_weight), F32P), _p(_f32(vis_weight), F32P),
                           _p(_f32(max_screen), F32P), ctypes.c_float(min_opacity), ctypes.c_float(max_bound),
                           _p(c, F32P), ctypes.c_float(split_at_screen_size), _p(table, F32P))
    assert rc == 0
    return table[:n]


def refine_split(transforms, sh, raw_opac, parents, children, screen, split_at_screen_size, min_opacity,
                 empty_rows=()):
    """Split of every parent into itself and its child row, plus filler rows
    (train.rs:2142-2283); returns updated copies."""
    L = lib()
    t, o = _f32(transforms).copy(), _f32(raw_opac).copy()
    n = t.shape[0]
    shf = _f32(np.asarray(sh, np.float32).reshape(n, -1)).copy()
    par = np.ascontiguousarray(parents, np.int32)
    ch = np.ascontiguousarray(children, np.int32)
    emp = np.ascontiguousarray(empty_rows, np.int32)
    scr = _f32(screen) if screen is not None else np.zeros(1, np.float32)
    I32P = ctypes.POINTER(ctypes.c_int32)
    rc = L.or_refine_split(_p(t, F32P), _p(shf, F32P), ctypes.c_uint32(shf.shape[1]), _p(o, F32P),
                           ctypes.c_uint32(len(par)), _p(par if len(par) else np.zeros(1, np.int32), I32P),
                           _p(ch if len(ch) else np.zeros(1, np.int32), I32P), _p(scr, F32P),
                           ctypes.c_float(split_at_screen_size), ctypes.c_float(min_opacity),
                           ctypes.c_uint32(len(emp)), _p(emp if len(emp) else np.zeros(1, np.int32), I32P))
    assert rc == 0
    return t, shf.reshape(np.asarray(sh).shape), o


def min_scale(transforms, view_cams, factor):
    """compute_min_scale (train.rs:353-387); view_cams [V, 4] = centre xyz, 1/max(focal, 1e-6)."""
    t = _f32(transforms)
    cams = _f32(view_cams)
    out = np.zeros(t.shape[0], np.float32)
    lib().or_min_scale(ctypes.c_uint32(t.shape[0]), _p(t, F32P), _p(cams, F32P), ctypes.c_uint32(cams.shape[0]),
                       ctypes.c_float(factor), _p(out, F32P))
    return out


def fold_min_scale(transforms, raw_opac, min_scale):
    """fold_min_scale (gaussian_splats.rs:165-188) on copies."""
    t = _f32(transforms).copy()
    o = _f32(raw_opac).copy()
    lib().or_fold_min_scale(ctypes.c_uint32(t.shape[0]), _p(t, F32P), _p(o, F32P), _p(_f32(min_scale), F32P))
    return t, o


def opacity_decay(raw_opac, amount):
    o = _f32(raw_opac).copy()
    lib().or_opacity_decay(ctypes.c_uint32(o.shape[0]), _p(o, F32P), ctypes.c_float(amount))
    return o


def splitmix_shuffle(n: int, seed: int) -> np.ndarray:
    keys = np.empty(n, np.uint32)
    lib().or_splitmix_shuffle(_p(keys, U32P), ctypes.c_uint64(n), ctypes.c_uint64(seed))
    return keys


def expf(x):
    x = _f32(x)
    y = np.empty_like(x)
    lib().or_expf_batch(_p(x, F32P), _p(y, F32P), ctypes.c_size_t(x.size))
    return y


def logf(x):
    x = _f32(x)
    y = np.empty_like(x)
    lib().or_logf_batch(_p(x, F32P), _p(y, F32P), ctypes.c_size_t(x.size))
    return y


def f16_roundtrip(x):
    x = _f32(x)
    h = np.empty(x.shape, np.uint16)
    back = np.empty_like(x)
    lib().or_f16_batch(_p(x, F32P), _p(h, U16P), _p(back, F32P), ctypes.c_size_t(x.size))
    return h, back


def render_forward(cam, cfg, splats, bg=(0.0, 0.0, 0.0), min_scale=None):
    """Projection + binning + rasterize forward, all on the CPU (with the Mip
    3D-filter floor when ``min_scale`` is given and cfg.has_min_scale is set)."""
    proj = project(cam, cfg, splats.transforms, splats.sh, splats.raw_opac, min_scale)
    binning = bin(cam, proj)
    pre_offsets = binning["tile_offsets"].copy()
    fwd = raster_fwd(cam, bg, proj, binning, splats.n)
    after = dict(binning)
    after["tile_offsets"] = fwd["tile_offsets"]
    return dict(proj=proj, binning=binning, binning_after=after, tile_offsets_pre=pre_offsets, **fwd)


def pack_view(pixels, alpha_mode: int = 0):
    """view_to_packed_data (scene.rs:113-161): u8 [H, W] or [H, W, C] with
    C in 1..4 -> (u32 [H, W], has_alpha).  alpha_mode 1 = transparent."""
    px = np.ascontiguousarray(pixels, dtype=np.uint8)
    if px.ndim == 2:
        px = px[..., None]
    h, w, c = px.shape
    out = np.zeros((h, w), np.uint32)
    rc = lib().or_pack_view(_p(px, U8P), ctypes.c_uint32(w), ctypes.c_uint32(h), ctypes.c_uint32(c),
                            ctypes.c_int32(alpha_mode), _p(out, U32P))
    assert rc == 0
    return out, c in (2, 4)


def ply_encode(transforms, sh, raw_opac):
    """PLY vertex rows [N, 14 + 3 rest] f32 (export.rs:393-417); sh [N, C, 3]."""
    t, o = _f32(transforms), _f32(raw_opac)
    s = _f32(np.asarray(sh, np.float32))
    n, coeffs = t.shape[0], s.shape[1]
    degree = int(round(coeffs ** 0.5)) - 1
    out = np.zeros((max(n, 1), 14 + 3 * (coeffs - 1)), np.float32)
    rc = lib().or_ply_encode(ctypes.c_uint32(n), ctypes.c_int32(degree), _p(t, F32P), _p(s, F32P), _p(o, F32P),
                             _p(out, F32P))
    assert rc == 0
    return out[:n]


def set_num_threads(n: int) -> int:
    """Threads for the OpenMP loops; returns the count now in effect."""
    lib().or_set_num_threads(ctypes.c_int(int(n)))
    return int(lib().or_max_threads())
