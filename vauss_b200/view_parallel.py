"""View-parallel training over several GPUs of one node.

The reference trains on one device (its multi-view steps sum the dense
gradients of several renders before one Adam step, the RasterPass::
BackwardDense path of crates/splat-train/src/train.rs:1516-1587).  Here every
rank holds a full replica of the splats, renders its own views, accumulates
the dense per-splat gradient rows [N, 10 + 3(d+1)^2 + 1] of those views, and
one all-reduce (sum) over the ranks gives every replica the gradient of the
whole batch; each rank then runs the same deterministic 8-bit-moment Adam, so
the replicas stay bit-identical.

Two exchanges are available.  With a `PeerGroup` (the GPU path) the ranks'
gradient rows, view counts and parameter replicas live in buffers every rank
maps over NVLink: after a device barrier each rank runs the 8-bit-moment Adam
on its shard of the splats only (vs_adam_q8_peer), summing the rows of the
ranks that saw each splat straight from their memory and storing the new
parameters into every replica, and a second barrier ends the step.  Each
view writes compact rows of its own (vs_vjp_compact: 16 floats, the SH
gradient left as the colour gradient, plus the camera position and the view's
bit in a per-splat mask) and the owners rebuild the SH gradient; the sums run
over (rank, view) in order, bit for bit those of one dense row accumulated
over the same views (`compact_rows=False` keeps dense rows per rank).  Without
one, the dense gradient and the view counts go through one flat all-reduce
(`exchange`, injectable so the host logic runs with gloo ranks on the CPU) and
every rank runs the full replicated Adam.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Sequence

import numpy as np
import torch
import torch.distributed as dist

from . import _native as N
from . import ops
from .peer import PeerGroup
from .trainer import SceneBatch, Splats, SplatTrainer, TrainConfig, TrainStepStats


MAX_VIEW_SLOTS = 32  # compact rows: view slots per rank and step (bits of the per-splat mask)


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
                 peer: PeerGroup | None = None, compact_rows: bool = True, **kw):
        assert config.optimizer == "q8", "the view-parallel path steps the 8-bit m+v optimizer"
        super().__init__(config, device, **kw)
        self.exchange = exchange
        self.peer = peer
        self.compact_rows = compact_rows  # with a peer group: one compact row slot per view
        self.flat = None
        self.peer_set = None

    @staticmethod
    def shard_of(n: int, world: int, rank: int) -> tuple[int, int]:
        """Rank's splats [begin, end): contiguous runs of whole 256-splat blocks."""
        blocks = (n + 255) // 256
        b0, b1 = rank * blocks // world, (rank + 1) * blocks // world
        return b0 * 256, min(b1 * 256, n)

    def adopt(self, splats: Splats) -> Splats:
        """With a peer group, copies the splats (identical on every rank) into
        replicas that all ranks map and returns them; step_views must be given
        the returned splats.  Without one, returns `splats` unchanged."""
        if self.peer is None:
            return splats
        g, n = self.peer, splats.num_splats
        nc = splats.sh_coeffs.shape[1]
        width = 10 + nc * 3 + 1
        f32 = torch.float32
        addr_t, addr_sh, addr_o = g.alloc(n * 10, f32), g.alloc(n * nc * 3, f32), g.alloc(n, f32)
        addr_g = g.alloc(n * width, f32, zero=True)  # dense rows, or compact rows of up to 3 views
        addr_v = g.alloc(n, f32, zero=True)
        addr_c = g.alloc(4 * MAX_VIEW_SLOTS, f32, zero=True)  # camera position of each view slot
        addr_m = g.alloc(n, torch.int32, zero=True)  # view slots that saw each splat (compact rows)
        t = g.local(addr_t, n * 10, f32).view(n, 10)
        sh = g.local(addr_sh, n * nc * 3, f32).view(n, nc, 3)
        o = g.local(addr_o, n, f32)
        t.copy_(splats.transforms)
        sh.copy_(splats.sh_coeffs.float())
        o.copy_(splats.raw_opacities)
        self._grads = g.local(addr_g, n * width, f32).view(n, width)
        self._vis = g.local(addr_v, n, f32)
        self._cams = g.local(addr_c, 4 * MAX_VIEW_SLOTS, f32).view(MAX_VIEW_SLOTS, 4)
        self._mask = g.local(addr_m, n, torch.int32)
        self._addr_dense = addr_g
        self._addr_compact, self._compact_slots = addr_g, (n * width) // (n * N.COMPACT_ROW) if n else 0
        ps = N.PeerSet()
        ps.world, ps.rank = g.world, g.rank
        for r in range(g.world):
            ps.grads[r], ps.vis[r], ps.cams[r], ps.view_masks[r] = addr_g[r], addr_v[r], addr_c[r], addr_m[r]
            ps.transforms[r], ps.sh_coeffs[r], ps.raw_opacities[r] = addr_t[r], addr_sh[r], addr_o[r]
        self.peer_set = ps
        self.shard = self.shard_of(n, g.world, g.rank)
        m = self.shard[1] - self.shard[0]
        self.optim = dict(t=ops.Q8Moments(m * 10, self.device), sh=ops.Q8Moments(m * nc * 3, self.device),
                          o=ops.Q8Moments(m, self.device), time=0)
        self.record = None
        self._resident = t.data_ptr()
        return Splats(t, sh, o)

    def _compact_rows(self, views: int, n: int) -> list[torch.Tensor]:
        """Each view slot's [n, 16] compact rows; the dense-row buffer holds up
        to 3 slots, more take a peer buffer of their own, allocated by all
        ranks together the first time a step has that many views."""
        if views > self._compact_slots:
            addr = self.peer.alloc(views * n * N.COMPACT_ROW, torch.float32, zero=True)
            self._addr_compact, self._compact_slots = addr, views
            self._compact_local = self.peer.local(addr, views * n * N.COMPACT_ROW, torch.float32)
        base = self._compact_local if self._addr_compact is not self._addr_dense else self._grads.view(-1)
        return [base[v * n * N.COMPACT_ROW:(v + 1) * n * N.COMPACT_ROW] for v in range(views)]

    def step_views(self, batches: Sequence[SceneBatch], splats: Splats, hook=None) -> tuple[Splats, TrainStepStats]:
        """One optimizer step over this rank's views.  ``hook(name)``, when
        given, runs after each stage (render, loss, raster_bwd, vjp_dense per
        view; then barrier_rows, optimizer, barrier_params or exchange,
        optimizer), where a benchmark records CUDA events."""
        c = self.config
        mark = hook or (lambda name: None)
        peer = self.peer
        if peer is not None and self.peer_set is None:
            raise RuntimeError("call adopt(splats) before step_views with a peer group")
        if peer is not None and splats.transforms.data_ptr() != self._resident:
            raise RuntimeError("step_views needs the splats returned by adopt()")
        if self.optim is None:
            self._init_state(splats)
        self.step_count += 1
        n = splats.num_splats
        width = 10 + splats.sh_coeffs.shape[1] * 3 + 1
        # every rank renders the same number of views per step, so all ranks
        # agree on the row format (and allocate compact slots together)
        compact = peer is not None and self.compact_rows and 1 <= len(batches) <= MAX_VIEW_SLOTS
        if peer is not None:
            # rows are overwritten where vis is 0 (or the view's mask bit is
            # clear), so only the counts and masks are cleared
            grads, vis = self._grads, self._vis
            vis.zero_()
            if compact:
                self._mask.zero_()
                crows = self._compact_rows(len(batches), n)
        else:
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
        # host targets go up on a side stream, overlapped with the renders
        gts, ready = [], []
        host = [b for b in batches if b.img_packed.device != self.device]
        if host:
            cur = torch.cuda.current_stream(self.device)
            if self._copy_stream is None:
                self._copy_stream = torch.cuda.Stream(self.device)
            self._copy_stream.wait_stream(cur)  # the previous step no longer reads the buffers
        for i, b in enumerate(batches):
            if b.img_packed.device == self.device:
                gts.append(b.img_packed)
                ready.append(None)
                continue
            dst = self._buf(f"gt{i}", tuple(b.img_packed.shape), b.img_packed.dtype)
            with torch.cuda.stream(self._copy_stream):
                dst.copy_(b.img_packed, non_blocking=True)
            gts.append(dst)
            ready.append(self._copy_stream.record_event())
        for slot, (b, gt, ev) in enumerate(zip(batches, gts, ready)):
            cam = b.camera
            cfg = ops.render_cfg(splats.sh_degree, mip=c.render_mode_mip, background=self.background(),
                                 has_min_scale=splats.min_scale is not None)
            out = ops.render(cam, cfg, splats.transforms, splats.sh_coeffs, splats.raw_opacities,
                             min_scale=splats.min_scale, frame=self.frame,
                             out_img=self._buf("img", (cam.height, cam.width, 4), torch.float32),
                             visible=self._buf("visible", (n,), torch.float32))
            mark("render")
            if ev is not None:
                torch.cuda.current_stream(self.device).wait_event(ev)
            loss = ops.image_loss(out.out_img, gt, c.l1_weight, c.ssim_loss_weight)
            losses.append(loss.loss.clone())
            mark("loss")
            vc = ops.rasterize_bwd(out.frame, out.out_img, loss.dl_dpred,
                                   self._buf("v_combined", (max(n, 1), 10), torch.float32))
            mark("raster_bwd")
            if compact:
                ops.vjp_compact(out.frame, cfg, splats.transforms, splats.sh_coeffs, splats.raw_opacities, vc,
                                crows[slot], refine, self._cams[slot], self._mask, slot, min_scale=splats.min_scale,
                                visible=out.visible, vis_accum=vis)
            else:
                ops.vjp_dense(out.frame, cfg, splats.transforms, splats.sh_coeffs, splats.raw_opacities, vc, grads,
                              refine, min_scale=splats.min_scale, visible=out.visible, vis_accum=vis)
            mark("vjp_dense")
            num_visible += out.num_visible
            num_isect += out.num_intersections
        if peer is None:
            self.exchange(self.flat)
            mark("exchange")
        self.optim["time"] += 1
        time = self.optim["time"]
        o = self.optim
        opac_reg = c.opacity_reg / max(n, 1) if self.step_count <= c.total_train_iters // 3 else 0.0
        q8 = ops.q8_cfg(time, self.transforms_lr(), c.lr_coeffs_dc, c.lr_coeffs_dc / c.lr_coeffs_sh_scale, c.lr_opac,
                        opac_reg=opac_reg, eps=c.adam_epsilon,
                        noise_scale=c.mean_noise_weight * self.lr_unit() * self.median_scale,
                        noise_limit=self.median_scale, noise_seed=int(self.rng.integers(0, 2 ** 32)))
        if peer is not None:
            ps = self.peer_set
            ps.row_format, ps.views = (1, len(batches)) if compact else (0, 0)
            for r in range(peer.world):
                ps.grads[r] = (self._addr_compact if compact else self._addr_dense)[r]
            peer.barrier()  # every rank's rows and counts are complete
            mark("barrier_rows")
            ops.adam_q8_peer(splats.sh_degree, n, self.shard[0], self.shard[1], self.peer_set, o["t"], o["sh"],
                             o["o"], q8, device=self.device)
            mark("optimizer")
            peer.barrier()  # every replica holds the new parameters
            mark("barrier_params")
        else:
            ops.adam_q8_dense(splats.sh_degree, splats.transforms, splats.sh_coeffs, splats.raw_opacities, grads,
                              o["t"], o["sh"], o["o"], q8, opacities=None, visible=vis)
            mark("optimizer")
        loss_total = torch.stack(losses).sum() if losses else torch.zeros((), device=self.device)
        stats = TrainStepStats(loss=loss_total, num_visible=num_visible, num_intersections=num_isect,
                               lr_mean=float(self.transforms_lr()[0]), lr_coeffs=c.lr_coeffs_dc, lr_opac=c.lr_opac)
        return splats, stats
