"""Torch-facing wrappers of the C ABI, mirroring the reference's operator
traits (SplatOps / LossOps / SplatBwdOps / ProjectUpdateOps / QuantMomentOps /
HousekeepOps).  Tensors are CUDA tensors in the reference layouts; the kernels
run on the current torch stream of the tensors' device.  torch is used here
for device memory and streams only; every computation is a call into
libvauss_b200.so.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np
import torch

from . import _native as N
from .camera import Camera

_contexts: dict[int, "Context"] = {}


def _ptr(t: torch.Tensor | None):
    if t is None:
        return None
    assert t.is_cuda and t.is_contiguous(), "vauss_b200 ops take contiguous CUDA tensors"
    return ctypes.c_void_p(t.data_ptr())


class Context:
    """One vs_ctx per device (its stream follows torch's current stream)."""

    def __init__(self, device: int):
        self.device = device
        self.lib = N.lib()
        h = ctypes.c_void_p()
        with torch.cuda.device(device):
            N.check(None, self.lib.vs_ctx_create(device, ctypes.byref(h)))
        self.h = h

    def bind(self) -> "Context":
        s = torch.cuda.current_stream(self.device).cuda_stream
        N.check(self.h, self.lib.vs_ctx_set_stream(self.h, ctypes.c_void_p(s)))
        return self

    def check(self, status: int):
        N.check(self.h, status)

    @property
    def workspace_bytes(self) -> int:
        return int(self.lib.vs_ctx_workspace_bytes(self.h))

    @property
    def launch_count(self) -> int:
        return int(self.lib.vs_ctx_launch_count(self.h))

    def __del__(self):
        try:
            if getattr(self, "h", None):
                self.lib.vs_ctx_destroy(self.h)
        except Exception:
            pass


def context(device: int | torch.device | None = None) -> Context:
    if device is None:
        device = torch.cuda.current_device()
    if isinstance(device, torch.device):
        device = device.index if device.index is not None else torch.cuda.current_device()
    ctx = _contexts.get(device)
    if ctx is None:
        ctx = _contexts[device] = Context(device)
    return ctx.bind()


def render_cfg(sh_degree: int, mip: bool = True, sh_half: bool = False, background=(0.0, 0.0, 0.0),
               log_scale_offset: float = 0.0, has_min_scale: bool = False) -> N.RenderCfg:
    c = N.RenderCfg()
    c.mip, c.sh_degree, c.sh_half, c.has_min_scale = int(mip), int(sh_degree), int(sh_half), int(has_min_scale)
    c.log_scale_offset = float(log_scale_offset)
    for i in range(3):
        c.bg[i] = float(background[i])
    return c


class Frame:
    """Per-render state (vs_frame): the reference's RenderOutput internals and
    GaussianBackwardState (src/render_aux.rs:16-86, bwd/burn_glue.rs:205-229)."""

    def __init__(self, ctx: Context):
        self.ctx = ctx
        h = ctypes.c_void_p()
        ctx.check(ctx.lib.vs_frame_create(ctx.h, ctypes.byref(h)))
        self.h = h
        self.counts = N.RenderCounts()

    def __del__(self):
        try:
            if getattr(self, "h", None):
                self.ctx.lib.vs_frame_destroy(self.h)
        except Exception:
            pass

    @property
    def num_visible(self) -> int:
        return int(self.counts.num_visible)

    @property
    def num_intersections(self) -> int:
        return int(self.counts.num_intersections)

    def field(self, name: str) -> torch.Tensor:
        """A copy of one frame buffer as a CUDA tensor (u32 fields as int32)."""
        p = ctypes.c_void_p()
        n = ctypes.c_uint64()
        fid = N.FIELDS[name]
        self.ctx.check(self.ctx.lib.vs_frame_buffer(self.h, fid, ctypes.byref(p), ctypes.byref(n)))
        dtype = torch.float32 if name in ("depths", "projected", "opacities", "max_radius") else torch.int32
        out = torch.empty(max(int(n.value), 1), dtype=dtype, device=f"cuda:{self.ctx.device}")
        self.ctx.check(self.ctx.lib.vs_frame_copy(self.h, fid, _ptr(out), ctypes.c_uint64(int(n.value) * 4)))
        return out[: int(n.value)]


@dataclass
class RenderOutput:
    """SplatOps::render output for a training pass (src/render_aux.rs:16-86)."""

    out_img: torch.Tensor  # [H, W, 4] f32
    visible: torch.Tensor  # [N] f32
    frame: Frame

    @property
    def num_visible(self) -> int:
        return self.frame.num_visible

    @property
    def num_intersections(self) -> int:
        return self.frame.num_intersections


def render(camera: Camera, cfg: N.RenderCfg, transforms: torch.Tensor, sh_coeffs: torch.Tensor,
           raw_opacities: torch.Tensor, min_scale: torch.Tensor | None = None, frame: Frame | None = None,
           out_img: torch.Tensor | None = None, visible: torch.Tensor | None = None) -> RenderOutput:
    """Training render forward (SplatOps::render, crates/splat-train-render/src/lib.rs:53-115)."""
    ctx = context(transforms.device)
    n = transforms.shape[0]
    assert transforms.shape == (n, 10) and raw_opacities.shape == (n,)
    assert sh_coeffs.shape[0] == n and sh_coeffs.shape[2] == 3 and sh_coeffs.shape[1] == (cfg.sh_degree + 1) ** 2
    assert (sh_coeffs.dtype == torch.float16) == bool(cfg.sh_half)
    frame = frame or Frame(ctx)
    dev = transforms.device
    if out_img is None:
        out_img = torch.empty(camera.height, camera.width, 4, dtype=torch.float32, device=dev)
    if visible is None:
        visible = torch.empty(n, dtype=torch.float32, device=dev)
    cam = camera.to_c()
    ctx.check(ctx.lib.vs_render_forward(ctx.h, frame.h, ctypes.byref(cam), ctypes.byref(cfg), n, _ptr(transforms),
                                        _ptr(sh_coeffs), _ptr(raw_opacities), _ptr(min_scale), _ptr(out_img),
                                        _ptr(visible), ctypes.byref(frame.counts)))
    return RenderOutput(out_img, visible, frame)


def render_image(camera: Camera, cfg: N.RenderCfg, transforms: torch.Tensor, sh_coeffs: torch.Tensor,
                 raw_opacities: torch.Tensor, min_scale: torch.Tensor | None = None, frame: Frame | None = None,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    """Inference render (render_splats with RasterPass::Forward,
    crates/splat-train-render/src/gaussian_splats.rs:511-527): packed RGBA8
    [H, W] (int32 storage of the u32 words, r in the low byte)."""
    ctx = context(transforms.device)
    n = transforms.shape[0]
    assert transforms.shape == (n, 10) and raw_opacities.shape == (n,)
    assert sh_coeffs.shape[0] == n and sh_coeffs.shape[2] == 3 and sh_coeffs.shape[1] == (cfg.sh_degree + 1) ** 2
    assert (sh_coeffs.dtype == torch.float16) == bool(cfg.sh_half)
    frame = frame or Frame(ctx)
    if out is None:
        out = torch.empty(camera.height, camera.width, dtype=torch.int32, device=transforms.device)
    cam = camera.to_c()
    ctx.check(ctx.lib.vs_render_image(ctx.h, frame.h, ctypes.byref(cam), ctypes.byref(cfg), n, _ptr(transforms),
                                      _ptr(sh_coeffs), _ptr(raw_opacities), _ptr(min_scale), _ptr(out),
                                      ctypes.byref(frame.counts)))
    return out


def render_stages(camera: Camera, cfg: N.RenderCfg, transforms, sh_coeffs, raw_opacities, frame: Frame, out_img,
                  visible, min_scale=None, hook=None) -> RenderOutput:
    """``render`` as its three stages (project, bin, rasterize); ``hook(name)``
    runs after each (the benchmark records CUDA events there)."""
    ctx = frame.ctx.bind()
    cam = camera.to_c()
    ctx.check(ctx.lib.vs_render_project(ctx.h, frame.h, ctypes.byref(cam), ctypes.byref(cfg), transforms.shape[0],
                                        _ptr(transforms), _ptr(sh_coeffs), _ptr(raw_opacities), _ptr(min_scale),
                                        ctypes.byref(frame.counts)))
    if hook:
        hook("project")
    ctx.check(ctx.lib.vs_render_bin(ctx.h, frame.h))
    if hook:
        hook("bin")
    ctx.check(ctx.lib.vs_render_rasterize(ctx.h, frame.h, _ptr(out_img), _ptr(visible)))
    if hook:
        hook("raster_fwd")
    return RenderOutput(out_img, visible, frame)


@dataclass
class LossOutput:
    loss: torch.Tensor  # [] f32 on device
    partials: torch.Tensor  # [3, tiles]
    dl_dpred: torch.Tensor | None  # [H, W, 4]


def image_loss(pred: torch.Tensor, gt_packed: torch.Tensor, l1_weight: float, ssim_weight: float,
               with_grad: bool = True, out: LossOutput | None = None) -> LossOutput:
    """Fused L1 + SSIM loss with its gradient (LossOps, crates/splat-train-loss/src/lib.rs:1306-1389).
    The reference training objective is ``l1_weight = 1 - w, ssim_weight = -w``."""
    ctx = context(pred.device)
    h, w = pred.shape[0], pred.shape[1]
    assert pred.shape == (h, w, 4) and gt_packed.shape == (h, w)
    tiles = ((w + 15) // 16) * ((h + 15) // 16)
    if out is None:
        out = LossOutput(torch.empty((), dtype=torch.float32, device=pred.device),
                         torch.empty(3, tiles, dtype=torch.float32, device=pred.device),
                         torch.empty(h, w, 4, dtype=torch.float32, device=pred.device) if with_grad else None)
    ctx.check(ctx.lib.vs_loss(ctx.h, h, w, _ptr(pred), _ptr(gt_packed), ctypes.c_float(l1_weight),
                              ctypes.c_float(ssim_weight), _ptr(out.partials), _ptr(out.loss), _ptr(out.dl_dpred)))
    return out


def rasterize_bwd(frame: Frame, out_img: torch.Tensor, v_output: torch.Tensor,
                  v_combined: torch.Tensor | None = None) -> torch.Tensor:
    """SplatBwdOps::rasterize_bwd: v_combined [V, 10] (src/bwd/render_bwd.rs:27-155)."""
    ctx = frame.ctx.bind()
    v = frame.num_visible
    if v_combined is None or v_combined.shape[0] < v:
        v_combined = torch.empty(max(v, 1), 10, dtype=torch.float32, device=out_img.device)
    ctx.check(ctx.lib.vs_rasterize_backward(ctx.h, frame.h, _ptr(out_img), _ptr(v_output), _ptr(v_combined)))
    return v_combined[:v]


def adam_coefficients(time: int, beta1: float = 0.9, beta2: float = 0.999):
    """(beta1, beta2, inv1, inv2) for 1-based step ``time`` in f32, with
    beta^t by binary exponentiation in f32 as the reference's f32::powi
    (crates/splat-train/src/optim.rs:268-277)."""
    def powi(b: np.float32, e: int) -> np.float32:
        r = np.float32(1.0)
        base = np.float32(b)
        while e:
            if e & 1:
                r = np.float32(r * base)
            e >>= 1
            if e:
                base = np.float32(base * base)
        return r
    b1, b2 = np.float32(beta1), np.float32(beta2)
    inv1 = np.float32(np.float32(1.0) / np.float32(np.float32(1.0) - powi(b1, time)))
    inv2 = np.float32(np.float32(1.0) / np.float32(np.float32(1.0) - powi(b2, time)))
    return float(b1), float(b2), float(inv1), float(inv2)


def project_update(frame: Frame, cfg: N.RenderCfg, transforms, sh_coeffs, raw_opacities, v_combined, w_t,
                   lr_scale, w_o, adam: N.AdamCfg, color_dir, v_refine, grad_sq, variance=None, first_step=False,
                   min_scale=None):
    """ProjectUpdateOps::project_update (src/bwd/project_update.rs:84-224): in place."""
    ctx = frame.ctx.bind()
    lr = (ctypes.c_float * 10)(*[float(x) for x in lr_scale])
    ctx.check(ctx.lib.vs_project_update(ctx.h, frame.h, ctypes.byref(cfg), transforms.shape[0], _ptr(transforms),
                                        _ptr(sh_coeffs), _ptr(raw_opacities), _ptr(min_scale), _ptr(v_combined),
                                        _ptr(w_t), lr, _ptr(w_o), ctypes.byref(adam), _ptr(color_dir),
                                        _ptr(v_refine), _ptr(grad_sq), _ptr(variance), int(bool(first_step))))


def sh_step(params_f16, color_dir, grad_rows, codes, scales, variance, lr_scale, beta, factor, inv1, inv2, eps, lr,
            round_seed):
    """QuantMomentOps::step_moment on the colour path (quant_kernels.rs:277-376): in place."""
    ctx = context(params_f16.device)
    n = params_f16.shape[0]
    rw = int(np.prod(params_f16.shape[1:]))
    lrs = (ctypes.c_float * rw)(*[float(x) for x in lr_scale])
    ctx.check(ctx.lib.vs_sh_step(ctx.h, n, rw, _ptr(params_f16), _ptr(color_dir), _ptr(grad_rows), _ptr(codes),
                                 _ptr(scales), _ptr(variance), lrs, ctypes.c_float(beta), ctypes.c_float(factor),
                                 ctypes.c_float(inv1), ctypes.c_float(inv2), ctypes.c_float(eps),
                                 ctypes.c_float(lr), ctypes.c_uint32(round_seed)))


class Q8Moments:
    """8-bit m and v for one parameter tensor of ``count`` values (256-value blocks)."""

    def __init__(self, count: int, device):
        blocks = (count + 255) // 256
        self.m_codes = torch.full((count,), 128, dtype=torch.uint8, device=device)
        self.v_codes = torch.zeros(count, dtype=torch.uint8, device=device)
        self.m_scales = torch.zeros(blocks, dtype=torch.float32, device=device)
        self.v_scales = torch.zeros(blocks, dtype=torch.float32, device=device)

    def c(self) -> N.Q8Tensor:
        t = N.Q8Tensor()
        t.m_codes, t.v_codes = self.m_codes.data_ptr(), self.v_codes.data_ptr()
        t.m_scales, t.v_scales = self.m_scales.data_ptr(), self.v_scales.data_ptr()
        return t


def q8_cfg(time: int, lr_transforms, lr_sh_dc: float, lr_sh_rest: float, lr_opac: float, opac_reg: float = 0.0,
           eps: float = 1e-15, noise_scale: float = 0.0, noise_limit: float = 0.0, noise_seed: int = 0,
           beta1: float = 0.9, beta2: float = 0.999) -> N.Q8Cfg:
    b1, b2, inv1, inv2 = adam_coefficients(time, beta1, beta2)
    c = N.Q8Cfg()
    c.beta1, c.beta2, c.inv1, c.inv2, c.epsilon = b1, b2, inv1, inv2, float(eps)
    for i in range(10):
        c.lr_transforms[i] = float(lr_transforms[i])
    c.lr_sh_dc, c.lr_sh_rest, c.lr_opac, c.opac_reg = float(lr_sh_dc), float(lr_sh_rest), float(lr_opac), float(opac_reg)
    c.seed = int(time) & 0xffffffff
    c.noise_scale, c.noise_limit, c.noise_seed = float(noise_scale), float(noise_limit), int(noise_seed) & 0xffffffff
    return c


def step_q8(frame: Frame, cfg: N.RenderCfg, transforms, sh_coeffs, raw_opacities, v_combined, mom_t: Q8Moments,
            mom_sh: Q8Moments, mom_o: Q8Moments, q8: N.Q8Cfg, visible=None, refine_norm=None, vis_count=None,
            max_screen=None, min_scale=None):
    """Single-view fused VJP + 8-bit-moment Adam + refine statistics + mean noise (in place);
    ``min_scale`` is the Mip 3D-filter floor the frame was rendered with, if any."""
    ctx = frame.ctx.bind()
    ctx.check(ctx.lib.vs_step_q8(ctx.h, frame.h, ctypes.byref(cfg), transforms.shape[0], _ptr(transforms),
                                 _ptr(sh_coeffs), _ptr(raw_opacities), _ptr(min_scale), _ptr(v_combined),
                                 mom_t.c(), mom_sh.c(),
                                 mom_o.c(), ctypes.byref(q8), _ptr(visible), _ptr(refine_norm), _ptr(vis_count),
                                 _ptr(max_screen)))


def vjp_dense(frame: Frame, cfg: N.RenderCfg, transforms, sh_coeffs, raw_opacities, v_combined, grads, refine,
              min_scale=None, visible=None, vis_accum=None):
    """Accumulates one view's dense gradient rows [N, 10 + 3(d+1)^2 + 1] (multi-view path)."""
    ctx = frame.ctx.bind()
    ctx.check(ctx.lib.vs_vjp_dense(ctx.h, frame.h, ctypes.byref(cfg), transforms.shape[0], _ptr(transforms),
                                   _ptr(sh_coeffs), _ptr(raw_opacities), _ptr(min_scale), _ptr(v_combined),
                                   _ptr(grads), _ptr(refine), _ptr(visible), _ptr(vis_accum)))


def vjp_compact(frame: Frame, cfg: N.RenderCfg, transforms, sh_coeffs, raw_opacities, v_combined, rows, refine,
                cam_out, view_mask, slot: int = 0, min_scale=None, visible=None, vis_accum=None):
    """View `slot`'s compact gradient rows [N, 16] (transforms | raw opacity | colour gradient), its bit
    in view_mask [N] u32 and the camera position the VJP used (cam_out [4]); the shard owner rebuilds
    the SH gradient (adam_q8_peer with PeerSet.row_format = 1)."""
    ctx = frame.ctx.bind()
    ctx.check(ctx.lib.vs_vjp_compact(ctx.h, frame.h, ctypes.byref(cfg), transforms.shape[0], _ptr(transforms),
                                     _ptr(sh_coeffs), _ptr(raw_opacities), _ptr(min_scale), _ptr(v_combined),
                                     _ptr(rows), _ptr(refine), _ptr(visible), _ptr(vis_accum), _ptr(view_mask),
                                     int(slot), _ptr(cam_out)))


def min_scale(transforms: torch.Tensor, view_cams: torch.Tensor, factor: float,
              out: torch.Tensor | None = None) -> torch.Tensor:
    """Mip-Splatting 3D-filter floor per splat (compute_min_scale, crates/splat-train/src/train.rs:353-387);
    ``view_cams`` [V, 4] f32 rows (centre x, y, z, 1 / max(focal_px, 1e-6))."""
    ctx = context(transforms.device)
    n = transforms.shape[0]
    out = torch.empty(n, dtype=torch.float32, device=transforms.device) if out is None else out
    cams = view_cams.contiguous()
    ctx.check(ctx.lib.vs_min_scale(ctx.h, n, _ptr(transforms), _ptr(cams), cams.shape[0], ctypes.c_float(factor),
                                   _ptr(out)))
    return out


def fold_min_scale(transforms: torch.Tensor, raw_opacities: torch.Tensor, min_scale: torch.Tensor):
    """Splats::bake_min_scale (gaussian_splats.rs:165-188, 394-402): folds the floor into the
    log-scales and raw opacities in place."""
    ctx = context(transforms.device)
    ctx.check(ctx.lib.vs_fold_min_scale(ctx.h, transforms.shape[0], _ptr(transforms), _ptr(raw_opacities),
                                        _ptr(min_scale)))


def adam_q8_dense(sh_degree: int, transforms, sh_coeffs, raw_opacities, grads, mom_t: Q8Moments,
                  mom_sh: Q8Moments, mom_o: Q8Moments, q8: N.Q8Cfg, opacities=None, visible=None):
    ctx = context(transforms.device)
    ctx.check(ctx.lib.vs_adam_q8_dense(ctx.h, transforms.shape[0], sh_degree, _ptr(transforms), _ptr(sh_coeffs),
                                       _ptr(raw_opacities), _ptr(grads), mom_t.c(), mom_sh.c(), mom_o.c(),
                                       ctypes.byref(q8), _ptr(opacities), _ptr(visible)))


def adam_q8_peer(sh_degree: int, num_splats: int, splat_begin: int, splat_end: int, peers: N.PeerSet,
                 mom_t: Q8Moments, mom_sh: Q8Moments, mom_o: Q8Moments, q8: N.Q8Cfg, device=None):
    """Sharded Q8 Adam over the replicas of a view-parallel step (vs_adam_q8_peer);
    `peers` holds every rank's buffers as raw device addresses."""
    ctx = context(device)
    ctx.check(ctx.lib.vs_adam_q8_peer(ctx.h, num_splats, sh_degree, splat_begin, splat_end, ctypes.byref(peers),
                                      mom_t.c(), mom_sh.c(), mom_o.c(), ctypes.byref(q8)))


def gather_stats(refine_norm, vis_count, max_screen, refine_weight, visible, radius):
    ctx = context(refine_norm.device)
    ctx.check(ctx.lib.vs_gather_stats(ctx.h, refine_norm.shape[0], _ptr(refine_norm), _ptr(vis_count),
                                      _ptr(max_screen), _ptr(refine_weight), _ptr(visible), _ptr(radius)))


def noise_means(transforms, opacities, visible, scale: float, limit: float, seed: int):
    ctx = context(transforms.device)
    ctx.check(ctx.lib.vs_noise_means(ctx.h, transforms.shape[0], _ptr(transforms), _ptr(opacities), _ptr(visible),
                                     ctypes.c_float(scale), ctypes.c_float(limit), ctypes.c_uint32(seed)))


def radix_sort_pairs(keys: torch.Tensor, values: torch.Tensor, key_bits: int = 32):
    ctx = context(keys.device)
    ctx.check(ctx.lib.vs_radix_sort_pairs(ctx.h, _ptr(keys), _ptr(values), keys.numel(), key_bits))


def scan_inclusive(data: torch.Tensor) -> int:
    ctx = context(data.device)
    total = torch.zeros(1, dtype=torch.int64, device=data.device)
    ctx.check(ctx.lib.vs_scan_inclusive(ctx.h, _ptr(data), data.numel(), _ptr(total)))
    return int(total.item())


def math_probe(which: str, x: torch.Tensor) -> torch.Tensor:
    ctx = context(x.device)
    y = torch.empty_like(x)
    modes = {"exp": 0, "log": 1, "sqrt_rn": 2, "sqrt_ieee": 3, "rcp_rn": 4, "rcp_ieee": 5}
    ctx.check(ctx.lib.vs_math_probe(ctx.h, modes[which], _ptr(x), _ptr(y), x.numel()))
    return y
