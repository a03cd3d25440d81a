"""View-parallel training over several GPUs of one node.

The reference trains on one device (its multi-view steps sum the dense
gradients of several renders before one Adam step, the RasterPass::
BackwardDense path of crates/splat-train/src/train.rs:1516-1587).  Here every
rank holds a full replica of the splats, renders its own views, accumulates
the dense per-splat gradient rows [N, 10 + 3(d+1)^2 + 1] of those views, and
one all-reduce (sum) over the ranks gives every replica the gradient of the
whole batch; each rank then runs the same deterministic 8-bit-moment Adam, so
the replicas stay bit-identical.

The per-step exchange is one flat buffer: the dense gradient followed by the
per-splat count of views that saw the splat (the mean-noise gate).  torch.
distributed (NCCL over NVLink on the GPUs) carries it; `exchange` is injectable
so the host logic can be exercised with gloo ranks on the CPU.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Sequence

import numpy as np
import torch
import torch.distributed as dist

from . import ops
from .trainer import SceneBatch, Splats, SplatTrainer, TrainConfig, TrainStepStats


def views_for_rank(num_views: int, rank: int, world: int, step: int, per_rank: int) -> list[int]:
    """The global batch of step `step` is views [step*world*per_rank, ...) mod
    num_views; rank r takes its contiguous share."""
    start = (step * world + rank) * per_rank
    return [(start + i) % num_views for i in range(per_rank)]


def all_reduce_sum(t: torch.Tensor):
    dist.all_reduce(t, op=dist.ReduceOp.SUM)


@dataclass
class ExchangeLayout:
    n: int
    width: int

    @property
    def size(self) -> int:
        return self.n * self.width + self.n

    def views(self, flat: torch.Tensor):
        g = flat[: self.n * self.width].view(self.n, self.width)
        vis = flat[self.n * self.width:]
        return g, vis


class ViewParallelTrainer(SplatTrainer):
    """SplatTrainer whose step takes this rank's views and all-reduces the
    dense gradient before the replicated Q8 Adam step."""

    def __init__(self, config: TrainConfig, device, exchange: Callable[[torch.Tensor], None] = all_reduce_sum,
                 **kw):
        assert config.optimizer == "q8", "the view-parallel path steps the 8-bit m+v optimizer"
        super().__init__(config, device, **kw)
        self.exchange = exchange
        self.flat = None

    def step_views(self, batches: Sequence[SceneBatch], splats: Splats) -> tuple[Splats, TrainStepStats]:
        c = self.config
        if self.optim is None:
            self._init_state(splats)
        self.step_count += 1
        n = splats.num_splats
        width = 10 + splats.sh_coeffs.shape[1] * 3 + 1
        layout = ExchangeLayout(n, width)
        if self.flat is None or self.flat.numel() != layout.size:
            self.flat = torch.zeros(layout.size, dtype=torch.float32, device=self.device)
        else:
            self.flat.zero_()
        grads, vis = layout.views(self.flat)
        refine = self._buf("refine_dense", (n,), torch.float32)
        refine.zero_()
        losses = []
        num_visible = num_isect = 0
        if self.frame is None:
            self.frame = ops.Frame(ops.context(self.device))
        for b in batches:
            gt = b.img_packed if b.img_packed.device == self.device else b.img_packed.to(self.device,
                                                                                         non_blocking=True)
            cam = b.camera
            cfg = ops.render_cfg(splats.sh_degree, mip=c.render_mode_mip, background=self.background())
            out = ops.render(cam, cfg, splats.transforms, splats.sh_coeffs, splats.raw_opacities, frame=self.frame,
                             out_img=self._buf("img", (cam.height, cam.width, 4), torch.float32),
                             visible=self._buf("visible", (n,), torch.float32))
            loss = ops.image_loss(out.out_img, gt, c.l1_weight, c.ssim_loss_weight)
            losses.append(loss.loss.clone())
            vc = ops.rasterize_bwd(out.frame, out.out_img, loss.dl_dpred,
                                   self._buf("v_combined", (max(n, 1), 10), torch.float32))
            ops.vjp_dense(out.frame, cfg, splats.transforms, splats.sh_coeffs, splats.raw_opacities, vc, grads,
                          refine, visible=out.visible, vis_accum=vis)
            num_visible += out.num_visible
            num_isect += out.num_intersections
        self.exchange(self.flat)
        self.optim["time"] += 1
        time = self.optim["time"]
        o = self.optim
        opac_reg = c.opacity_reg / max(n, 1) if self.step_count <= c.total_train_iters // 3 else 0.0
        q8 = ops.q8_cfg(time, self.transforms_lr(), c.lr_coeffs_dc, c.lr_coeffs_dc / c.lr_coeffs_sh_scale, c.lr_opac,
                        opac_reg=opac_reg, eps=c.adam_epsilon,
                        noise_scale=c.mean_noise_weight * self.lr_unit() * self.median_scale,
                        noise_limit=self.median_scale, noise_seed=int(self.rng.integers(0, 2 ** 32)))
        ops.adam_q8_dense(splats.sh_degree, splats.transforms, splats.sh_coeffs, splats.raw_opacities, grads,
                          o["t"], o["sh"], o["o"], q8, opacities=None, visible=vis)
        loss_total = torch.stack(losses).sum() if losses else torch.zeros((), device=self.device)
        stats = TrainStepStats(loss=loss_total, num_visible=num_visible, num_intersections=num_isect,
                               lr_mean=float(self.transforms_lr()[0]), lr_coeffs=c.lr_coeffs_dc, lr_opac=c.lr_opac)
        return splats, stats
