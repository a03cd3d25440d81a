"""Refinement: prune, replace and grow splats (densification).

Host side of SplatTrainer::refine (crates/splat-train/src/train.rs:
1779-2104) and refine_splats (:2110-2300).  The GPU builds one per-splat
decision table (vs_refine_table), read back once; from it the host picks the
dead rows, the bounds of the surviving splats and the parents (replacements of
the dead weighted by opacity x visibility, screen-oversized splats, and
growth toward the budget weighted by the refine statistic); vs_refine_split
then splits every parent into itself and a child written into a dead row or
an appended one, the children's optimizer moments are zeroed
(vs_q8_reset_rows), and the opacities decay (vs_opacity_decay).

Differences from the reference, on purpose: parents are sampled with numpy's
weighted sampling without replacement (the reference's rand crate draws a
different stream), and parents are processed in index order (the reference
iterates a hash set).  The periodic Morton re-ordering of the splats
(train.rs:2017-2020) and the Mip-Splatting floor refresh (:2067-2083, only for
training images below 0.3 MP) are not part of this path.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np
import torch

from . import _native as N
from . import ops

MIN_OPACITY = 1.0 / 255.0  # train.rs:36
BOUND_PERCENTILE = 0.8  # train.rs:34
GROWTH_FULL_AT = 0.8  # train.rs:189
AUTO_MAX_SPLATS = 1_200_000  # train.rs:306-344
AUTO_MAX_SPLATS_LOCAL = 2_000_000
AUTO_MAX_SPLATS_MAX = 8_000_000
AUTO_MAX_SPLATS_MAX_BASE = 2_000_000
FAR_RADIUS, FAR_SHARE_FLOOR, FAR_BUDGET_GAIN = 2.0, 0.05, 10.0
MIN_PIXELS_PER_SPLAT = 30


@dataclass
class Bounds:
    center: np.ndarray
    extent: np.ndarray  # half sizes

    @staticmethod
    def from_means(means: np.ndarray, percentile: float = BOUND_PERCENTILE) -> "Bounds":
        """bounds_from_pos (crates/splat-train/src/splat_init.rs:167-195)."""
        lo, hi = np.empty(3, np.float32), np.empty(3, np.float32)
        for a in range(3):
            v = means[:, a][np.isfinite(means[:, a])]
            if v.size == 0:
                return Bounds(np.zeros(3, np.float32), np.ones(3, np.float32))
            n = v.size
            i_lo = int((1.0 - percentile) / 2.0 * n)
            i_hi = min(n - 1, int((1.0 + percentile) / 2.0 * n))
            part = np.partition(v, (i_lo, i_hi))
            lo[a], hi[a] = part[i_lo], part[i_hi]
        return Bounds((lo + hi) / 2, (hi - lo) / 2)


@dataclass
class RefineStats:
    """crates/splat-train/src/msg.rs RefineStats."""

    num_added: int
    num_split_oversized: int
    num_split_high_grad: int
    num_pruned: int
    num_pruned_non_finite: int
    num_relocated: int
    total_splats: int


def weighted_sample(rng: np.random.Generator, weights: np.ndarray, k: int) -> list[int]:
    """k distinct indices drawn with probability proportional to the weights,
    non-finite or negative weights counting as 0 (multinomial.rs:1-28)."""
    w = np.where(np.isfinite(weights) & (weights >= 0), weights, 0.0).astype(np.float64)
    k = min(int(k), int(np.count_nonzero(w)))
    if k <= 0:
        return []
    return rng.choice(w.size, size=k, replace=False, p=w / w.sum()).tolist()


class Refiner:
    """Refine state of one trainer: scene bounds, budget and the RNG."""

    def __init__(self, config, bounds: Bounds, rng: np.random.Generator, train_pixels: int = 0,
                 view_centers: np.ndarray | None = None):
        self.config = config
        self.bounds = bounds
        self.rng = rng
        self.train_pixels = int(train_pixels)
        self.view_centers = view_centers
        self.far_share: float | None = None
        self.growth_start_count: int | None = None

    # ---- budget (train.rs:626-687) ----
    def measure_far_share(self, means: np.ndarray) -> float:
        if self.view_centers is None or len(self.view_centers) == 0:
            return 0.0
        c = self.view_centers.mean(axis=0)
        d = np.sort(np.linalg.norm(self.view_centers - c, axis=1))
        spread = d[(len(d) - 1) * 95 // 100]
        far = np.linalg.norm(means - c, axis=1) > FAR_RADIUS * max(spread, 1e-6)
        return float(far.sum()) / max(len(means), 1)

    def auto_budget(self) -> int:
        far = self.far_share or 0.0
        by_pixels = 2 ** 32 - 1 if self.train_pixels == 0 else self.train_pixels // MIN_PIXELS_PER_SPLAT
        scale = 1.0 + FAR_BUDGET_GAIN * max(far - FAR_SHARE_FLOOR, 0.0)
        base, ceiling = ((AUTO_MAX_SPLATS_MAX_BASE, AUTO_MAX_SPLATS_MAX) if self.config.max_budget
                         else (AUTO_MAX_SPLATS, AUTO_MAX_SPLATS_LOCAL))
        return int(min(int(base * scale), ceiling, by_pixels))

    def splat_cap(self, n0: int) -> int:
        c = self.config
        if c.max_splats > 0:
            return c.max_splats
        end = min(c.growth_stop_iter, c.total_train_iters)
        steps = max(end - c.growth_start_iter, 0)
        return max(min(int(n0 * 1.05 ** (steps / 100.0)), self.auto_budget()), n0)

    # ---- the refine step ----
    def refine(self, it: int, splats, record, optim: dict, device) -> tuple:
        """Returns (splats, stats, new record); `optim` holds the Q8 moments
        (t, sh, o) and is updated in place."""
        c = self.config
        ctx = ops.context(device)
        n = splats.num_splats
        sh_width = splats.sh_coeffs.shape[1] * 3
        sh_half = splats.sh_coeffs.dtype == torch.float16
        cfg = N.RefineCfg()
        cfg.min_opacity = MIN_OPACITY
        cfg.max_bound = float(self.bounds.extent.max()) * 100.0
        for a in range(3):
            cfg.center[a] = float(self.bounds.center[a])
        cfg.split_at_screen_size = c.split_at_screen_size
        table = torch.empty(max(n, 1), 8, dtype=torch.float32, device=device)
        ctx.check(ctx.lib.vs_refine_table(ctx.h, n, ops._ptr(splats.transforms), ops._ptr(splats.sh_coeffs),
                                          sh_width, int(sh_half), ops._ptr(splats.raw_opacities),
                                          ops._ptr(record.refine_norm), ops._ptr(record.vis_count),
                                          ops._ptr(record.max_screen), ctypes.byref(cfg), ops._ptr(table)))
        host = table[:n].cpu().numpy()  # the one readback
        if self.far_share is None and c.max_splats == 0:
            self.far_share = self.measure_far_share(host[:, 5:8])
        dead = np.flatnonzero(host[:, 0] != 0).tolist()
        if len(dead) == n:
            dead = []
        dead_mask = np.zeros(n, bool)
        dead_mask[dead] = True
        alive = n - len(dead)
        num_non_finite = int((host[:, 1] != 0).sum())
        new_bounds = Bounds.from_means(host[~dead_mask, 5:8])

        def alive_col(k):
            return np.where(dead_mask, 0.0, host[:, k])

        split = []  # insertion-ordered set
        seen = set()

        def add(ind):
            if ind not in seen:
                seen.add(ind)
                split.append(ind)
                return True
            return False

        for i in weighted_sample(self.rng, alive_col(2), len(dead)) if dead else []:
            add(i)
        pre = len(split)
        if c.split_at_screen_size > 0:
            n0 = self.growth_start_count if self.growth_start_count is not None else alive
            budget = max(self.splat_cap(n0) - (alive + len(split)), 0)
            for ind in np.flatnonzero(alive_col(3) != 0):
                if budget == 0:
                    break
                if add(int(ind)):
                    budget -= 1
        num_oversized = len(split) - pre
        pre = len(split)
        if c.growth_start_iter <= it < c.growth_stop_iter:
            if self.growth_start_count is None:
                self.growth_start_count = n
            n0 = float(self.growth_start_count)
            cap = float(self.splat_cap(int(n0)))
            start = float(c.growth_start_iter)
            full = max(min(GROWTH_FULL_AT * c.total_train_iters, float(c.growth_stop_iter)), start + 1.0)
            t = min(max((it - start) / (full - start), 0.0), 1.0)
            target = min(int(np.ceil(n0 * max(cap / max(n0, 1.0), 1.0) ** t)), int(cap))
            grow = max(target - (alive + len(split)), 0)
            if grow > 0:
                for i in weighted_sample(self.rng, alive_col(4), grow):
                    add(i)
        num_high_grad = len(split) - pre
        parents = sorted(split)
        splats = self._split(ctx, splats, optim, parents, dead, record.max_screen, sh_width, sh_half, it, device)
        self.bounds = new_bounds
        new_n = splats.num_splats
        stats = RefineStats(num_added=len(parents), num_split_oversized=num_oversized,
                            num_split_high_grad=num_high_grad, num_pruned=len(dead),
                            num_pruned_non_finite=num_non_finite, num_relocated=min(len(dead), len(parents)),
                            total_splats=new_n)
        return splats, stats

    def _split(self, ctx, splats, optim, parents, dead, screen, sh_width, sh_half, it, device):
        c = self.config
        from .trainer import Splats
        n = splats.num_splats
        r = len(parents)
        empty = dead[r:] if len(dead) > r else []
        dead = dead[:r]
        filled = len(dead)
        extra = r - filled
        t, sh, o = splats.transforms, splats.sh_coeffs, splats.raw_opacities
        if extra > 0:  # appended rows, written by the split below
            t = torch.cat([t, torch.zeros(extra, 10, dtype=t.dtype, device=device)])
            sh = torch.cat([sh, torch.zeros(extra, *sh.shape[1:], dtype=sh.dtype, device=device)])
            o = torch.cat([o, torch.zeros(extra, dtype=o.dtype, device=device)])
        new_n = n + extra
        children = dead + list(range(n, new_n))
        i32 = lambda v: torch.tensor(v if v else [0], dtype=torch.int32, device=device)
        par_d, ch_d, emp_d = i32(parents), i32(children), i32(empty)
        ctx.check(ctx.lib.vs_refine_split(ctx.h, new_n, ops._ptr(t), ops._ptr(sh), sh_width, int(sh_half), ops._ptr(o),
                                          r, ops._ptr(par_d), ops._ptr(ch_d),
                                          ops._ptr(screen) if c.split_at_screen_size > 0 else None,
                                          c.split_at_screen_size, MIN_OPACITY, len(empty), ops._ptr(emp_d)))
        if optim is not None:
            reset = parents + dead + empty
            self._reset_moments(ctx, optim, reset, extra, sh_width, device)
        minus = c.opac_decay * (1.0 - min(max(it / max(c.total_train_iters, 1), 0.0), 1.0))
        ctx.check(ctx.lib.vs_opacity_decay(ctx.h, new_n, ops._ptr(o), minus))
        return Splats(t, sh, o)

    @staticmethod
    def _reset_moments(ctx, optim, rows, extra, sh_width, device):
        rows_d = torch.tensor(rows if rows else [0], dtype=torch.int32, device=device)
        for key, width in (("t", 10), ("sh", sh_width), ("o", 1)):
            m: ops.Q8Moments = optim[key]
            if extra > 0:  # appended rows: zero codes; new blocks: zero scales
                count = m.m_codes.numel() + extra * width
                blocks = (count + 255) // 256
                m.m_codes = torch.cat([m.m_codes, torch.full((extra * width,), 128, dtype=torch.uint8, device=device)])
                m.v_codes = torch.cat([m.v_codes, torch.zeros(extra * width, dtype=torch.uint8, device=device)])
                nb = blocks - m.m_scales.numel()
                if nb > 0:
                    m.m_scales = torch.cat([m.m_scales, torch.zeros(nb, device=device)])
                    m.v_scales = torch.cat([m.v_scales, torch.zeros(nb, device=device)])
            if rows:
                ctx.check(ctx.lib.vs_q8_reset_rows(ctx.h, m.c(), width, len(rows), ops._ptr(rows_d)))
