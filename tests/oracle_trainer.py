"""SplatTrainer.step restated with the CPU oracle (test infrastructure).

Shares the trainer's host-side schedule (learning rates, background and noise
seeds from the same generator) and replaces every device call with the
oracle's restatement, so whole training steps can be compared.
"""
from __future__ import annotations

import numpy as np

import oracle
from vauss_b200 import ops
from vauss_b200.scenes import SplatSet
from vauss_b200.trainer import SplatTrainer, TrainConfig


def _q8_zero(count):
    blocks = (count + 255) // 256
    return [np.full(count, 128, np.uint8), np.zeros(count, np.uint8), np.zeros(blocks, np.float32),
            np.zeros(blocks, np.float32)]


class OracleTrainer(SplatTrainer):
    def __init__(self, config: TrainConfig, sp: SplatSet, **kw):
        super().__init__(config, "cpu", **kw)
        self.sp = SplatSet(sp.transforms.copy(), sp.sh.copy(), sp.raw_opac.copy())
        n = sp.n
        self.norm = np.zeros(n, np.float32)
        self.vis = np.zeros(n, np.float32)
        self.screen = np.zeros(n, np.float32)
        self.time = 0
        self.min_scale = None  # the Mip 3D-filter floor [N] f32, when set
        if config.optimizer == "q8":
            self.mom = {"t": _q8_zero(n * 10), "sh": _q8_zero(sp.sh.size), "o": _q8_zero(n)}
        else:
            c = sp.sh.shape[1]
            blocks = (n * c * 3 + 127) // 128
            self.w_t = np.zeros((n, 10), np.uint32)
            self.w_o = np.zeros(n, np.uint32)
            self.codes = np.full(blocks * 32, 0x80808080, np.uint32)
            self.scales = np.zeros(blocks, np.float32)
            self.variance = np.zeros(n, np.float32)
            self.sh_half = None

    def step_oracle(self, gt_packed: np.ndarray, cam) -> float:
        c = self.config
        self.step_count += 1
        bg = self.background()
        sp = self.sp
        n = sp.n
        half = c.optimizer == "reference" and self.sh_half is not None
        sh_now = self.sh_half.view(np.uint16) if half else sp.sh
        ms = self.min_scale
        cfg = oracle.make_cfg(sp.sh_degree, mip=c.render_mode_mip, sh_half=half, bg=bg, has_min_scale=ms is not None)
        r = oracle.render_forward(cam, cfg, SplatSet(sp.transforms, sh_now, sp.raw_opac), bg=bg, min_scale=ms)
        lo = oracle.loss_fwd(r["out_img"], gt_packed, c.l1_weight, c.ssim_loss_weight)
        dl = oracle.loss_bwd(r["out_img"], gt_packed, lo["coeffs"], c.l1_weight, c.ssim_loss_weight)
        vc = oracle.raster_bwd(cam, bg, r["proj"], r["binning_after"], r["out_img"], dl)
        self.time += 1
        time = self.time
        lr_t = self.transforms_lr()
        opac_reg = c.opacity_reg / max(n, 1) if self.step_count <= c.total_train_iters // 3 else 0.0
        noise_scale = c.mean_noise_weight * self.lr_unit() * self.median_scale
        noise_seed = int(self.rng.integers(0, 2 ** 32))
        b1, b2, inv1, inv2 = ops.adam_coefficients(time)
        if c.optimizer == "q8":
            grads, refine = oracle.vjp_dense(cam, cfg, sp.transforms, sp.sh, sp.raw_opac,
                                             r["proj"]["compact_from_global"], vc, min_scale=ms)
            if opac_reg:
                o = (np.float32(1) / (np.float32(1) + oracle.expf(-sp.raw_opac))).astype(np.float32)
                grads[:, -1] = (grads[:, -1] + np.float32(opac_reg) * o * (np.float32(1) - o)).astype(np.float32)
            width = grads.shape[1]
            wsh = width - 11
            res_t = oracle.adam_q8(sp.transforms, grads, width, 0, 10, *self.mom["t"], lr_t, 1.0, b1, b2, inv1, inv2,
                                   c.adam_epsilon, time ^ (10 << 24))
            lr_sh = np.float32([c.lr_coeffs_dc] * 3 + [c.lr_coeffs_dc / c.lr_coeffs_sh_scale] * (wsh - 3))
            res_s = oracle.adam_q8(sp.sh.reshape(n, -1), grads, width, 10, wsh, *self.mom["sh"], lr_sh, 1.0, b1, b2,
                                   inv1, inv2, c.adam_epsilon, time ^ (48 << 24))
            res_o = oracle.adam_q8(sp.raw_opac, grads, width, width - 1, 1, *self.mom["o"], np.float32([c.lr_opac]),
                                   1.0, b1, b2, inv1, inv2, c.adam_epsilon, time ^ (1 << 24))
            self.mom = {"t": list(res_t[1:]), "sh": list(res_s[1:]), "o": list(res_o[1:])}
            t = res_t[0].reshape(n, 10)
            sh = res_s[0].reshape(sp.sh.shape)
            op = res_o[0]
        else:
            pu = oracle.project_update(cam, cfg, sp.transforms, sh_now, sp.raw_opac, r["proj"]["compact_from_global"],
                                       vc, self.w_t, lr_t, self.w_o, b1, b2, inv1, inv2, c.adam_epsilon, c.lr_opac,
                                       opac_reg, time, min_scale=ms)
            refine = pu["refine"]
            self.w_t, self.w_o = pu["w_t"], pu["w_o"]
            gsq = pu["grad_sq"]
            vis_rows = r["proj"]["compact_from_global"] > 0
            if time == 1:
                self.variance = (gsq * (np.float32(1) - np.float32(b2))).astype(np.float32)
            else:
                upd = self.variance * np.float32(b2) + gsq * (np.float32(1) - np.float32(b2))
                self.variance = np.where(vis_rows, upd, self.variance).astype(np.float32)
            if self.sh_half is None:
                self.sh_half = sp.sh.astype(np.float16)
            nc = sp.sh.shape[1]
            lr_scale = np.repeat(np.float32([1.0] + [1.0 / c.lr_coeffs_sh_scale] * (nc - 1)), 3)
            p, self.codes, self.scales = oracle.sh_step_ref(
                self.sh_half.view(np.uint16), pu["color_dir"], r["proj"]["compact_from_global"], self.codes,
                self.scales, self.variance, lr_scale, b1, float(np.float32(1) - np.float32(b1)), inv1, inv2,
                c.adam_epsilon, c.lr_coeffs_dc, time)
            self.sh_half = p.view(np.float16).reshape(sp.sh.shape)
            t, op = pu["transforms"], pu["raw_opac"]
            sh = self.sh_half.astype(np.float32)
        if noise_scale != 0.0:
            t = oracle.noise_means(t, r["proj"]["opacities"], r["visible"], noise_scale, self.median_scale,
                                   noise_seed)
        self.norm, self.vis, self.screen = oracle.gather_stats(self.norm, self.vis, self.screen, refine, r["visible"],
                                                               r["proj"]["max_radius"])
        self.sp = SplatSet(t, sh.astype(np.float32) if c.optimizer == "q8" else sp.sh, op)
        if c.optimizer != "q8":
            self.sp = SplatSet(t, sp.sh, op)
        return lo["loss"]

    def sh_values(self) -> np.ndarray:
        if self.config.optimizer == "q8":
            return self.sp.sh
        return self.sh_half.astype(np.float32)
