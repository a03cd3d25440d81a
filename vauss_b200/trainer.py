"""Training-step driver mirroring the reference trainer's API.

``SplatTrainer.step(batch, splats) -> (splats, TrainStepStats)`` follows
crates/splat-train/src/train.rs:747-1685 (``SplatTrainer::step`` /
``step_inner``) for single-view 3DGS steps on the fused-update pass
(RasterPass::BackwardFusedUpdate, train.rs:1031-1037):

  render forward -> L1 + SSIM loss -> rasterizer backward -> optimizer ->
  refine statistics + low-opacity mean noise.

Two optimizers:
  * ``"reference"`` -- the reference's storage: packed 16/16 moments for
    transforms and opacity (project_update), f16 SH coefficients with an 8-bit
    first moment in 128-value blocks and one reduced f32 second moment per
    splat (crates/splat-train/src/optim.rs);
  * ``"q8"`` -- the benchmark configuration: f32 parameters, 8-bit first and
    second moments in 256-value blocks with fp32 absmax scales, all 59
    parameters per splat, one fused kernel.

Every tensor operation of the step is a call into libvauss_b200.so; torch
holds device memory and the stream.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np
import torch

from . import ops
from .camera import Camera


# train.rs:41, 347: the 3D-filter floor stops being refreshed after 90 % of
# training and applies only to training images of at most 300k pixels
MIN_SCALE_FREEZE_FRAC = 0.9
MIP_3D_FILTER_MAX_PIXELS = 300_000


@dataclass
class TrainConfig:
    """Trainer options (crates/splat-train/src/config.rs:7-351 defaults)."""

    total_train_iters: int = 30_000
    lr_mean: float = 1.6e-4
    lr_mean_end: float = 1.6e-6
    mean_noise_weight: float = 6.25
    lr_coeffs_dc: float = 2e-3
    lr_coeffs_sh_scale: float = 10.0
    lr_opac: float = 0.012
    lr_scale: float = 5e-3
    lr_rotation: float = 2e-3
    ssim_weight: float = 0.2
    opacity_reg: float = 0.005
    background_color: tuple = (0.0, 0.0, 0.0)
    background_noise_strength: float = 0.1
    render_mode_mip: bool = True
    optimizer: str = "q8"  # "q8" | "reference"
    adam_epsilon: float = 1e-15
    # refinement (config.rs:238-290)
    refine_every: int = 200
    growth_start_iter: int = 500
    growth_stop_iter: int = 15_000
    max_splats: int = 0
    max_budget: bool = False
    split_at_screen_size: float = 0.5
    opac_decay: float = 0.004
    # Mip-Splatting 3D filter (config.rs:300-306): a per-splat scale floor of
    # sqrt(factor) pixel sizes at the nearest training camera, set at each
    # refine while training images have at most 300k pixels; 0 disables it
    min_scale_factor: float = 0.1

    @property
    def l1_weight(self) -> float:
        """(1 - w) L1 - w SSIM (train.rs:1180-1184)."""
        return 1.0 - self.ssim_weight if self.ssim_weight > 0 else 1.0

    @property
    def ssim_loss_weight(self) -> float:
        return -self.ssim_weight if self.ssim_weight > 0 else 0.0


@dataclass
class SceneBatch:
    """One training view (crates/splat-train-dataset/src/scene.rs:165-191):
    packed RGBA8 ground truth [H, W] (host or device) and its camera."""

    img_packed: torch.Tensor
    camera: Camera
    view_index: int = 0
    has_alpha: bool = False
    alpha_mode: int = 0


@dataclass
class Splats:
    """Per-splat parameters on the device (gaussian_splats.rs:131-153)."""

    transforms: torch.Tensor  # [N, 10] f32
    sh_coeffs: torch.Tensor  # [N, C, 3] f32 (f16 after the first reference-mode SH step)
    raw_opacities: torch.Tensor  # [N] f32
    # Mip 3D-filter floor [N] f32, folded into scales and opacity at render
    # (gaussian_splats.rs:331-402); None = no floor
    min_scale: torch.Tensor | None = None

    @property
    def num_splats(self) -> int:
        return int(self.transforms.shape[0])

    @property
    def sh_degree(self) -> int:
        return int(round(math.sqrt(self.sh_coeffs.shape[1]))) - 1

    @staticmethod
    def from_numpy(sp, device) -> "Splats":
        return Splats(torch.from_numpy(np.ascontiguousarray(sp.transforms)).to(device),
                      torch.from_numpy(np.ascontiguousarray(sp.sh)).to(device),
                      torch.from_numpy(np.ascontiguousarray(sp.raw_opac)).to(device))


@dataclass
class TrainStepStats:
    """crates/splat-train/src/msg.rs:20-30: the loss stays on the device until read."""

    loss: torch.Tensor
    num_visible: int
    num_intersections: int
    lr_mean: float
    lr_coeffs: float
    lr_opac: float


@dataclass
class RefineRecord:
    """Refine accumulators gathered each step (housekeep.rs:15-39)."""

    refine_norm: torch.Tensor
    vis_count: torch.Tensor
    max_screen: torch.Tensor


class SplatTrainer:
    def __init__(self, config: TrainConfig, device, scene_extent: float = 1.0, median_scale: float = 0.01,
                 seed: int = 42):
        self.config = config
        self.device = torch.device(device)
        self.step_count = 0
        self.scene_extent = float(scene_extent)
        self.median_scale = float(median_scale)
        iters = config.total_train_iters
        self.lr_mean_decay = (config.lr_mean_end / config.lr_mean) ** (1.0 / iters) if iters > 1 else 1.0
        self.rng = np.random.default_rng(seed)
        self.frame: ops.Frame | None = None
        self.optim = None
        self.record: RefineRecord | None = None
        self._buffers = {}
        self._copy_stream = None
        self.refiner = None
        self.train_pixels = 0  # pixels of all training images (the refine budget limit); 0 = unlimited
        self.view_centers = None  # [V, 3] camera centres (far-share of the refine budget)
        self.view_cams = None  # [V, 4] f32 device rows (centre, 1 / focal px) for the 3D-filter floor

    def set_view_cams(self, cameras, train_pixels: int | None = None):
        """The training cameras (SplatTrainer::set_view_cams, train.rs:608-619):
        their centres and focal lengths set the 3D-filter floor and the refine
        budget's far share; ``train_pixels`` defaults to the sum of their
        image sizes."""
        centers = np.array([c.position for c in cameras], dtype=np.float32).reshape(-1, 3)
        inv_f = np.array([np.float32(1.0) / np.float32(max(c.fx, 1e-6)) for c in cameras], dtype=np.float32)
        rows = np.concatenate([centers, inv_f[:, None]], axis=1).astype(np.float32)
        self.view_centers = centers
        self.view_cams = torch.from_numpy(rows).to(self.device) if len(cameras) else None
        self.train_pixels = int(sum(c.width * c.height for c in cameras)) if train_pixels is None else train_pixels

    def floor_applies(self, it: int) -> bool:
        """train.rs:2040-2047: the floor is refreshed at a refine before 90 % of
        training, with view cameras, a positive factor and training images of at
        most 300k pixels."""
        c = self.config
        if c.min_scale_factor <= 0 or self.view_cams is None or self.view_cams.shape[0] == 0:
            return False
        per_view = self.train_pixels // max(self.view_cams.shape[0], 1)
        small = self.train_pixels == 0 or per_view <= MIP_3D_FILTER_MAX_PIXELS
        return it / max(c.total_train_iters, 1) < MIN_SCALE_FREEZE_FRAC and small

    # ---- refinement (train.rs:1779-2300; vauss_b200/refine.py) ----
    def should_refine(self, step: int) -> bool:
        """The training loop's refine schedule (crates/splat-brush/src/train.rs:1136)."""
        c = self.config
        return step > 0 and step % c.refine_every == 0 and step / max(c.total_train_iters, 1) <= 0.95

    def refine(self, it: int, splats: Splats):
        """Prune, replace and grow the splats; returns (splats, RefineStats).
        The optimizer moments follow the rows; the refine statistics restart."""
        from .refine import Bounds, Refiner
        if self.config.optimizer != "q8":
            raise NotImplementedError("refinement is implemented for the 8-bit-moment optimizer")
        if self.optim is None or self.record is None:
            raise RuntimeError("refine needs at least one training step first")
        # the floor is folded into the parameters first (train.rs:1806), so the
        # decisions see the splats' real sizes and opacities
        if splats.min_scale is not None:
            ops.fold_min_scale(splats.transforms, splats.raw_opacities, splats.min_scale)
            splats = Splats(splats.transforms, splats.sh_coeffs, splats.raw_opacities)
        if self.refiner is None:
            means = splats.transforms[:, :3].detach().cpu().numpy()
            self.refiner = Refiner(self.config, Bounds.from_means(means), self.rng, self.train_pixels,
                                   self.view_centers)
        splats, stats = self.refiner.refine(it, splats, self.record, self.optim, self.device)
        n = splats.num_splats
        dev = self.device
        self.record = RefineRecord(torch.zeros(n, device=dev), torch.zeros(n, device=dev), torch.zeros(n, device=dev))
        # a fresh floor against the new positions (train.rs:2040-2056)
        if self.floor_applies(it):
            splats = Splats(splats.transforms, splats.sh_coeffs, splats.raw_opacities,
                            ops.min_scale(splats.transforms, self.view_cams, self.config.min_scale_factor))
        return splats, stats

    # ---- learning rates (train.rs:859-904) ----
    def lr_unit(self) -> float:
        return self.config.lr_mean * self.lr_mean_decay ** (self.step_count - 1)

    def transforms_lr(self) -> np.ndarray:
        c = self.config
        lr_mean = self.lr_unit() * self.scene_extent
        fixed = np.array([0, 0, 0, c.lr_rotation, c.lr_rotation, c.lr_rotation, c.lr_rotation, c.lr_scale,
                          c.lr_scale, c.lr_scale], dtype=np.float32)
        cols = np.array([1, 1, 1, 0, 0, 0, 0, 0, 0, 0], dtype=np.float32)
        return (fixed + cols * np.float32(lr_mean)).astype(np.float32)

    def background(self) -> tuple:
        c = self.config
        base = np.asarray(c.background_color, dtype=np.float32)
        s = c.background_noise_strength
        if s <= 0:
            return tuple(np.clip(base, 0, 1).tolist())
        noise = self.rng.uniform(-s, s, size=3).astype(np.float32)
        return tuple(np.clip(base + noise, 0, 1).tolist())

    def _buf(self, name, shape, dtype):
        t = self._buffers.get(name)
        if t is None or tuple(t.shape) != tuple(shape) or t.dtype != dtype:
            t = self._buffers[name] = torch.empty(shape, dtype=dtype, device=self.device)
        return t

    def _init_state(self, splats: Splats):
        n = splats.num_splats
        dev = self.device
        self.record = RefineRecord(torch.zeros(n, device=dev), torch.zeros(n, device=dev), torch.zeros(n, device=dev))
        if self.config.optimizer == "q8":
            self.optim = dict(t=ops.Q8Moments(n * 10, dev), sh=ops.Q8Moments(splats.sh_coeffs.numel(), dev),
                              o=ops.Q8Moments(n, dev), time=0)
        else:
            c = splats.sh_coeffs.shape[1]
            blocks = (n * c * 3 + 127) // 128
            self.optim = dict(w_t=torch.zeros(n, 10, dtype=torch.int32, device=dev),
                              w_o=torch.zeros(n, dtype=torch.int32, device=dev),
                              codes=torch.full((blocks * 32,), 0x80808080 - (1 << 32), dtype=torch.int32, device=dev),
                              scales=torch.zeros(blocks, device=dev), variance=torch.zeros(n, device=dev), time=0)

    def step(self, batch: SceneBatch, splats: Splats) -> tuple[Splats, TrainStepStats]:
        c = self.config
        if self.optim is None:
            self._init_state(splats)
        self.step_count += 1
        cam = batch.camera
        gt = batch.img_packed
        gt_ready = None
        if gt.device != self.device:
            # Upload the target on a side stream: the loss is its first reader,
            # so the copy overlaps projection, sorting and compositing.  The
            # copy waits for the previous step (the last reader of the buffer).
            cur = torch.cuda.current_stream(self.device)
            if self._copy_stream is None:
                self._copy_stream = torch.cuda.Stream(self.device)
            dst = self._buf("gt", tuple(gt.shape), gt.dtype)
            self._copy_stream.wait_stream(cur)
            with torch.cuda.stream(self._copy_stream):
                dst.copy_(gt, non_blocking=True)
            gt_ready = self._copy_stream.record_event()
            gt = dst
        bg = self.background()
        n = splats.num_splats
        mode = c.optimizer
        cfg = ops.render_cfg(splats.sh_degree, mip=c.render_mode_mip,
                             sh_half=splats.sh_coeffs.dtype == torch.float16, background=bg,
                             has_min_scale=splats.min_scale is not None)
        if self.frame is None:
            self.frame = ops.Frame(ops.context(self.device))
        out = ops.render(cam, cfg, splats.transforms, splats.sh_coeffs, splats.raw_opacities,
                         min_scale=splats.min_scale, frame=self.frame,
                         out_img=self._buf("img", (cam.height, cam.width, 4), torch.float32),
                         visible=self._buf("visible", (n,), torch.float32))
        if gt_ready is not None:
            torch.cuda.current_stream(self.device).wait_event(gt_ready)
        loss = ops.image_loss(out.out_img, gt, c.l1_weight, c.ssim_loss_weight)
        vcomb = self._buf("v_combined", (max(n, 1), 10), torch.float32)
        vc = ops.rasterize_bwd(out.frame, out.out_img, loss.dl_dpred, vcomb)
        self.optim["time"] += 1
        time = self.optim["time"]
        lr_t = self.transforms_lr()
        opac_reg = c.opacity_reg / max(n, 1) if self.step_count <= c.total_train_iters // 3 else 0.0
        noise_scale = c.mean_noise_weight * self.lr_unit() * self.median_scale
        noise_seed = int(self.rng.integers(0, 2 ** 32))
        rec = self.record
        if mode == "q8":
            o = self.optim
            q8 = ops.q8_cfg(time, lr_t, c.lr_coeffs_dc, c.lr_coeffs_dc / c.lr_coeffs_sh_scale, c.lr_opac,
                            opac_reg=opac_reg, eps=c.adam_epsilon, noise_scale=noise_scale,
                            noise_limit=self.median_scale, noise_seed=noise_seed)
            ops.step_q8(out.frame, cfg, splats.transforms, splats.sh_coeffs, splats.raw_opacities, vc, o["t"],
                        o["sh"], o["o"], q8, visible=out.visible, refine_norm=rec.refine_norm,
                        vis_count=rec.vis_count, max_screen=rec.max_screen, min_scale=splats.min_scale)
        else:
            splats = self._reference_optimizer_step(out, cfg, splats, vc, lr_t, opac_reg, time, noise_scale,
                                                    noise_seed)
        stats = TrainStepStats(loss=loss.loss, num_visible=out.num_visible,
                               num_intersections=out.num_intersections, lr_mean=float(lr_t[0]),
                               lr_coeffs=c.lr_coeffs_dc, lr_opac=c.lr_opac)
        return splats, stats

    def _reference_optimizer_step(self, out, cfg, splats, vc, lr_t, opac_reg, time, noise_scale, noise_seed):
        c = self.config
        o = self.optim
        n = splats.num_splats
        b1, b2, inv1, inv2 = ops.adam_coefficients(time)
        adam = ops.N.AdamCfg(b1, b2, inv1, inv2, c.adam_epsilon, c.lr_opac, opac_reg, time)
        color_dir = self._buf("color_dir", (n + 1, 6), torch.float32)
        refine = self._buf("refine", (n,), torch.float32)
        gsq = self._buf("grad_sq", (n,), torch.float32)
        ops.project_update(out.frame, cfg, splats.transforms, splats.sh_coeffs, splats.raw_opacities, vc,
                           o["w_t"], lr_t, o["w_o"], adam, color_dir, refine, gsq, variance=o["variance"],
                           first_step=(time == 1), min_scale=splats.min_scale)
        # SH coefficients live in f16 from the first SH step on (optim.rs:424-436)
        if splats.sh_coeffs.dtype != torch.float16:
            splats = Splats(splats.transforms, splats.sh_coeffs.to(torch.float16), splats.raw_opacities,
                            splats.min_scale)
        nc = splats.sh_coeffs.shape[1]
        lr_scale = np.repeat(np.float32([1.0] + [1.0 / c.lr_coeffs_sh_scale] * (nc - 1)), 3)
        cfrom = out.frame.field("compact_from_global")
        ops.sh_step(splats.sh_coeffs, color_dir, cfrom, o["codes"], o["scales"], o["variance"], lr_scale, b1,
                    float(np.float32(1) - np.float32(b1)), inv1, inv2, c.adam_epsilon, c.lr_coeffs_dc, time)
        rec = self.record
        ops.gather_stats(rec.refine_norm, rec.vis_count, rec.max_screen, refine, out.visible,
                         out.frame.field("max_radius"))
        if noise_scale != 0.0:
            ops.noise_means(splats.transforms, out.frame.field("opacities"), out.visible, noise_scale,
                            self.median_scale, noise_seed)
        return splats
