#!/usr/bin/env python
"""Benchmark of the Gaussian-splat training step (fwd + bwd + Adam).

Workload (benchmark configuration 2, "full training iteration at scale"):
3,000,000 SH-degree-3 splats (means U[-5,5]^3, log-scales N(-4.5, 0.6),
opacity logits N(0, 1.5), DC colours U[0,1], higher bands N(0, 0.05)),
200 pinhole views of 1600x1060 (fx = fy = 1300) on a jittered sphere of
radius 8, one view per step per GPU, L1 + 0.2 D-SSIM against targets rendered
from a second seeded splat set (quantised to RGBA8), Adam with 8-bit
block-quantised first and second moments (256-value blocks, fp32 absmax).
Synthetic data stand in for the reference's capture datasets.

One step = project/sort/rasterize forward, fused loss forward+backward,
rasterizer backward, projection VJP + Adam + refine statistics + mean noise.
With N GPUs every rank trains its own view per step; the ranks' dense
gradient rows are read over NVLink peer memory by a sharded fused Adam that
stores the new parameters into every replica (weak scaling: one view per GPU
per step); value = views/s over the whole job = iterations/s at N = 1.

With --config 3 it runs benchmark configuration 3 instead: 6,000,000 splats
(configuration-2 distributions) and a fixed global batch of 8 views of
1920x1080 (fx = fy = 1600) per step, split evenly over 1, 2, 4 or 8 GPUs
(strong scaling; value = global-batch steps/s).  Every GPU count, one
included, runs the peer-memory view-parallel trainer.

With --config 4 it runs the sort/overlap stress (configuration 4, one GPU):
10,000,000 large splats, one 3840x2160 view; value = intersections/s through
intersect + radix sort + tile ranges.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference] [--config 2|3|4]
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "fwd+bwd+Adam iters/s @3M splats 1600×1060; raster fwd/bwd HBM GB/s vs peak"
N_SPLATS = 3_000_000
N_VIEWS = 200
N_TARGETS = 8


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=100)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--splats", type=int, default=None, help="default: 3M (config 2), 6M (config 3)")
    p.add_argument("--config", type=int, default=2, choices=[2, 3, 4])
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    a = p.parse_args()
    if a.splats is None:
        a.splats = {2: N_SPLATS, 3: 6_000_000, 4: 10_000_000}[a.config]
    return a


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# ---------------------------------------------------------------- clocks ----
class ClockSampler:
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu_id = gpu_id
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", self.gpu_id, f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            t0 = time.monotonic()  # the sampler needs a moment to come up
            while not self.lines and time.monotonic() - t0 < 5.0 and self.proc.poll() is None:
                time.sleep(0.02)
        except Exception:
            self.proc = None
        return self

    def mark(self, which):
        setattr(self, which, time.monotonic())

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.monotonic(), line.strip()))

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        rows = []
        t0, t1 = getattr(self, "start", None), getattr(self, "stop", None)
        for ts, l in self.lines:
            parts = [x.strip() for x in l.split(",")]
            if len(parts) < 7:
                continue
            try:
                rows.append((float(parts[0]), float(parts[1]), float(parts[2]), parts[3:7], ts))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        inside = [r for r in rows if t0 is not None and t1 is not None and t0 <= r[4] <= t1]
        loaded = inside or [r for r in rows if r[2] > 200.0] or rows
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in loaded for i in range(4) if r[3][i].lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in loaded), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(loaded), "in_timed_region": bool(inside)}


# ------------------------------------------------------------ workloads ----
def make_workload(n_splats: int, config: int = 2):
    from vauss_b200 import scenes
    if config == 3:
        sp, cams = scenes.config_multiview(seed=4, n=n_splats, views=8)
    else:
        sp, cams = scenes.config_train(seed=3, n=n_splats, views=N_VIEWS)
    tgt = scenes.random_splats(n_splats, 1003, mean_lo=-5.0, mean_hi=5.0, log_scale_mu=-4.5, log_scale_sigma=0.6,
                               opac_mu=0.0, opac_sigma=1.5, sh_degree=3)
    return sp, tgt, cams


# DRAM bytes (read + write) per launch of each stage's kernel, from one ncu
# capture of this workload (config 2 at 3M splats; profiles/<kernel>_config2_3M.md
# give the command; the optimizer's second term is vjp_rows_kernel from the
# same capture, taken before that kernel compacted its rows).  Below the
# algorithmic bytes for the raster kernels: L2 (126 MB) serves a projected row
# to the neighbouring tiles that gather it.  Only the dominant stage's figure
# goes into the bench line.
MEASURED_TRAFFIC_CONFIG2 = {"raster_bwd": 273.6e6, "raster_fwd": 142.5e6, "project": 700.7e6, "loss": 60.8e6,
                           "optimizer": 2.352e9 + 474.1e6}


def stage_bytes(name: str, n: int, v: int, i: int, p: int, t: int) -> float:
    """Algorithmic (compulsory) DRAM bytes of one launch of each stage:
    each logically required byte counted once, no cross-CTA reuse."""
    if name == "project":  # params 44 B + 3 per-splat outputs; SH 192 B + row 48 + id/depth/count 12 per visible
        return n * (44 + 12) + v * (192 + 48 + 12)
    if name == "bin":  # depth sort 4 passes x 16 B; emission 8 B, tile sort 2 passes x 16 B, ranges 4 B per isect
        return v * (4 * 16 + 12) + i * (8 + 2 * 16 + 4)
    if name == "raster_fwd":  # id 4 + row 48 gathered per isect; RGBA write per pixel; visible marks
        return i * 52 + p * 16 + v * 4 + t * 12
    if name == "loss":  # pred 16 + gt 4 read, dL/dpred 16 write per pixel
        return p * 36
    if name == "raster_bwd":  # id + row per isect; image + upstream grad per pixel; zeroed + accumulated grads
        return i * 52 + p * 32 + v * 80
    if name == "optimizer":  # params r+w 472, m/v codes r+w 236, scales, cfg map 4, stats 24, noise gate 8 per splat
        return n * (472 + 236 + 4 + 24 + 8 + 2 * 59 * 8 / 256) + v * 40
    return 0.0


def run_ours(args):
    import torch
    import torch.distributed as dist
    from vauss_b200 import ops, scenes
    from vauss_b200.trainer import SceneBatch, Splats, SplatTrainer, TrainConfig
    from vauss_b200.view_parallel import ViewParallelTrainer, views_for_rank

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        from datetime import timedelta
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device(f"cuda:{local}"))
    dev = torch.device(f"cuda:{local}")
    torch.cuda.set_device(dev)

    multiview = args.config == 3
    if multiview and 8 % world:
        raise SystemExit("config 3 splits its 8 views over 1, 2, 4 or 8 GPUs")
    sp, tgt, cams = make_workload(args.splats, args.config)
    splats = Splats.from_numpy(sp, dev)
    # targets: rendered from the second splat set, quantised to RGBA8
    tsplats = Splats.from_numpy(tgt, dev)
    cfg_t = ops.render_cfg(3, mip=True)
    if multiview:  # this rank's share of the fixed global batch
        per_rank = 8 // world
        views = [rank * per_rank + k for k in range(per_rank)]
    else:
        views = [(rank * N_TARGETS + k) % N_VIEWS for k in range(N_TARGETS)]
    targets = []
    for vi in views:
        out = ops.render(cams[vi], cfg_t, tsplats.transforms, tsplats.sh_coeffs, tsplats.raw_opacities)
        img = out.out_img[..., :3].clamp(0, 1).cpu().numpy()
        targets.append(torch.from_numpy(scenes.pack_rgba8(img).view(np.int32)).to(dev))
    del tsplats
    torch.cuda.synchronize()

    cfg = TrainConfig(optimizer="q8")
    median_scale = float(np.median(np.exp(sp.transforms[:, 7:10])))
    kw = dict(scene_extent=8.0, median_scale=median_scale)
    peer = None
    if world > 1 or multiview:
        from vauss_b200.peer import PeerGroup, gather_bytes_nccl
        gather = (lambda b: gather_bytes_nccl(b, dev)) if world > 1 else (lambda b: [b])
        peer = PeerGroup(dev, world, rank, gather)
        trainer = ViewParallelTrainer(cfg, dev, peer=peer, **kw)
        splats = trainer.adopt(splats)
    else:
        trainer = SplatTrainer(cfg, dev, **kw)

    def step(k, loader=None):
        if multiview:
            batches = ([loader.next_batch() for _ in views] if loader else
                       [SceneBatch(targets[j], cams[views[j]], views[j]) for j in range(len(views))])
            return trainer.step_views(batches, splats)
        vi = k % N_TARGETS
        b = loader.next_batch() if loader else SceneBatch(targets[vi], cams[views[vi]], views[vi])
        if world > 1:
            return trainer.step_views([b], splats)
        return trainer.step(b, splats)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    counts = {}
    for k in range(args.warmup):
        _, st0 = step(k)
        counts = {"visible": int(st0.num_visible), "intersections": int(st0.num_intersections)}
    barrier()
    # The timed region starts from this state; the per-stage profile and the
    # end-to-end leg restart from it too, so that all three measure the same
    # workload (training moves the splats, and the raster work grows with it).
    import copy
    moments = ("m_codes", "v_codes", "m_scales", "v_scales")
    snap = {"p": [x.clone() for x in (splats.transforms, splats.sh_coeffs, splats.raw_opacities)],
            "m": {k: [getattr(trainer.optim[k], a).clone() for a in moments] for k in ("t", "sh", "o")},
            "time": trainer.optim["time"], "step": trainer.step_count,
            "rng": copy.deepcopy(trainer.rng.bit_generator.state)}

    def restore():
        for dst, src in zip((splats.transforms, splats.sh_coeffs, splats.raw_opacities), snap["p"]):
            dst.copy_(src)
        for k in ("t", "sh", "o"):
            for a, src in zip(moments, snap["m"][k]):
                getattr(trainer.optim[k], a).copy_(src)
        trainer.optim["time"], trainer.step_count = snap["time"], snap["step"]
        trainer.rng.bit_generator.state = copy.deepcopy(snap["rng"])
        barrier()
    ctx = ops.context(dev)
    launches0 = ctx.launch_count
    gpu_uuid = str(torch.cuda.get_device_properties(dev).uuid)
    gpu_id = gpu_uuid if gpu_uuid.startswith("GPU-") else f"GPU-{gpu_uuid}"
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(gpu_id) as clk:
        barrier()
        clk.mark("start")
        e0.record(stream)
        for k in range(args.steps):
            step(args.warmup + k)
        e1.record(stream)
        barrier()
        clk.mark("stop")
    ms = e0.elapsed_time(e1)
    launches = (ctx.launch_count - launches0) // max(args.steps, 1)
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    value = (1 if multiview else world) * args.steps / (ms_max / 1e3)

    # ---- end to end through the public API: host GT in, loss out ----
    e2e = None
    if not args.no_e2e:
        from vauss_b200 import dataset
        # the views as decoded RGB host images: the staged loader copies one
        # (per view of the step) from pinned memory every step and packs it
        rgb = [tg.cpu().numpy().view(np.uint8).reshape(tg.shape[0], tg.shape[1], 4)[..., :3].copy()
               for tg in targets]
        loader = dataset.SceneLoader(
            dataset.Scene([dataset.SceneView(img, cams[vi]) for img, vi in zip(rgb, views)]), seed=rank,
            config=dataset.LoadDatasetConfig(max_scene_batch_cache_size=0), device=dev,
            hold=len(views) if multiview else 1)
        loss_host = torch.empty((), dtype=torch.float32).pin_memory()
        for k in range(args.warmup):  # untimed: first use of the host-input path
            _, st = step(k, loader=loader)
            loss_host.copy_(st.loss, non_blocking=True)
        restore()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        h2d0 = loader.h2d_bytes_total
        f0.record(stream)
        for k in range(args.steps):
            _, st = step(k, loader=loader)
            loss_host.copy_(st.loss, non_blocking=True)
        f1.record(stream)
        barrier()
        ems = f0.elapsed_time(f1)
        h2d_total = loader.h2d_bytes_total - h2d0
        loader.close()
        te = torch.tensor([ems], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e2e = {"value": (1 if multiview else world) * args.steps / (float(te.item()) / 1e3),
               "unit": "steps/s" if multiview else "iters/s",
               "h2d_bytes_per_step": int(round(h2d_total / max(args.steps, 1))), "d2h_bytes_per_step": 4,
               "feed": "SceneLoader (vs_feed): RGB8 views, pinned ring of 4, packed on the GPU, no cache",
               "api": ("ViewParallelTrainer.step_views (vs_render_forward, vs_loss, vs_rasterize_backward, "
                       "vs_vjp_dense, vs_peer_barrier, vs_adam_q8_peer)" if world > 1 else
                       "SplatTrainer.step (vs_render_forward, vs_loss, vs_rasterize_backward, vs_step_q8)")}

    # ---- per-stage device times (CUDA events on the launching stream) ----
    stages = None
    roofline = None
    if world == 1 and not multiview:
        restore()
        stages = profile_stages(trainer, splats, targets, cams, views, dev, reps=5)
        peak, which = peaks()
        n, v, i = splats.num_splats, stages.pop("_v"), stages.pop("_i")
        cam0 = cams[views[0]]
        p, tcount = cam0.width * cam0.height, cam0.num_tiles
        for name, d in stages.items():
            b = stage_bytes(name, n, v, i, p, tcount)
            d["gbs"] = b / (d["ms"] / 1e3) / 1e9
            d["alg_bytes"] = b
        dom = max(stages, key=lambda k: stages[k]["ms"])
        ach = stages[dom]["gbs"]
        roofline = {"bound": "hbm", "kernel": dom, "achieved": round(ach, 1), "peak": peak, "unit": "GB/s",
                    "frac": round(ach / peak, 4),
                    "traffic": (MEASURED_TRAFFIC_CONFIG2.get(dom) if n == N_SPLATS else None), "peak_source": which,
                    "note": "raster stages are FP32-issue bound; see profiles/ for issue utilisation"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and not multiview:
        cpu = cpu_baseline(sp, tgt, cams, views, gt=targets[0].cpu().numpy().view(np.uint32))

    if multiview:
        workload = dict(workload="config 3: 6M SH-3 splats, global batch of 8 views of 1920x1080 split over the "
                                 f"GPUs ({len(views)} per GPU), L1+0.2 D-SSIM, 8-bit m+v Adam (block 256)",
                        splats=splats.num_splats, width=1920, height=1080, views_per_step=8)
    else:
        workload = dict(workload="config 2: 3M SH-3 splats, 1600x1060, 1 view/step/GPU, L1+0.2 D-SSIM, "
                                 "8-bit m+v Adam (block 256)", splats=splats.num_splats, width=1600, height=1060,
                        views_per_step=world)
    out = {"metric": ("view-parallel steps/s @6M splats, 8 views of 1920×1080 per step" if multiview else METRIC),
           "value": round(value, 3), "unit": "steps/s" if multiview else "iters/s", "n_gpus": world,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 4),
           "higher_is_better": True, "scaling": "strong" if multiview else "weak", "vs_baseline": None,
           "dtype": "f32", "data": "synthetic",
           "config": {**workload, "optimizer": "q8",
                      "parallelism": (f"view-parallel x{world}: dense gradient rows read over NVLink peer "
                                      f"memory by a sharded fused Adam that stores to every replica"
                                      if world > 1 or multiview else "single GPU"),
                      "l2": ("inputs larger than L2 (params + moments ~%.1f GB)"
                             % (splats.num_splats * (236 + 122) / 1e9)), **counts},
           "gpu_launches": int(launches), "clocks": clk.summary()}
    if roofline:
        out["roofline"] = roofline
    if stages:
        out["stages"] = {k: {"ms": round(d["ms"], 4), "gbs": round(d["gbs"], 1)} for k, d in stages.items()}
    if cpu:
        out["cpu_baseline"] = cpu
    if e2e:
        out["e2e"] = {k: (round(v, 3) if isinstance(v, float) else v) for k, v in e2e.items()}
    if rank == 0:
        print(json.dumps(out), flush=True)
    if world == 1 and peer is not None:
        torch.cuda.synchronize(dev)
        peer.check()
        peer.close()
    if world > 1:
        dist.barrier()
        torch.cuda.synchronize(dev)
        dist.barrier()  # no rank's kernels touch peer buffers any more
        if peer is not None:
            peer.check()
            peer.close()
        torch.cuda.synchronize(dev)
        dist.barrier()
        dist.destroy_process_group()


def profile_stages(trainer, splats, targets, cams, views, dev, reps=5):
    """Per-stage device times of the single-view step with CUDA events: the
    median over `reps` steps, so that a host stall between two launches (which
    the events on the device timeline include) in one step does not count."""
    import torch
    from vauss_b200 import ops
    c = trainer.config
    stream = torch.cuda.current_stream(dev)
    acc = {}
    n = splats.num_splats
    frame = trainer.frame
    v = i = 0
    for r in range(reps):
        vi = r % len(targets)
        cam = cams[views[vi]]
        cfg = ops.render_cfg(3, mip=True, background=(0.0, 0.0, 0.0))
        evs = [("start", torch.cuda.Event(enable_timing=True))]
        evs[0][1].record(stream)

        def hook(name):
            e = torch.cuda.Event(enable_timing=True)
            e.record(stream)
            evs.append((name, e))
        img = trainer._buf("img", (cam.height, cam.width, 4), torch.float32)
        vis = trainer._buf("visible", (n,), torch.float32)
        out = ops.render_stages(cam, cfg, splats.transforms, splats.sh_coeffs, splats.raw_opacities, frame, img, vis,
                                hook=hook)
        loss = ops.image_loss(out.out_img, targets[vi], c.l1_weight, c.ssim_loss_weight)
        hook("loss")
        vc = ops.rasterize_bwd(out.frame, out.out_img, loss.dl_dpred,
                               trainer._buf("v_combined", (max(n, 1), 10), torch.float32))
        hook("raster_bwd")
        o = trainer.optim
        o["time"] += 1
        q8 = ops.q8_cfg(o["time"], trainer.transforms_lr(), c.lr_coeffs_dc, c.lr_coeffs_dc / c.lr_coeffs_sh_scale,
                        c.lr_opac, eps=c.adam_epsilon, noise_scale=1e-7, noise_limit=1e-3, noise_seed=r)
        rec = trainer.record
        ops.step_q8(out.frame, cfg, splats.transforms, splats.sh_coeffs, splats.raw_opacities, vc, o["t"], o["sh"],
                    o["o"], q8, visible=out.visible, refine_norm=rec.refine_norm, vis_count=rec.vis_count,
                    max_screen=rec.max_screen)
        hook("optimizer")
        torch.cuda.synchronize()
        for (a, ea), (b, eb) in zip(evs[:-1], evs[1:]):
            acc.setdefault(b, []).append(ea.elapsed_time(eb))
        v += out.num_visible / reps
        i += out.num_intersections / reps
    out = {k: {"ms": float(statistics.median(t))} for k, t in acc.items()}
    out["_v"] = v
    out["_i"] = i
    return out


# --------------------------------------------------- CPU baseline (oracle) ----
def oracle_step(sp, cam, gt, mom, time_step):
    """One full training step of the CPU oracle (the reference's algorithm
    restated on the host): the same stages as the GPU step."""
    import oracle
    from vauss_b200 import ops
    cfg = oracle.make_cfg(3, mip=True)
    r = oracle.render_forward(cam, cfg, sp)
    lo = oracle.loss_fwd(r["out_img"], gt, 0.8, -0.2)
    dl = oracle.loss_bwd(r["out_img"], gt, lo["coeffs"], 0.8, -0.2)
    vc = oracle.raster_bwd(cam, (0.0, 0.0, 0.0), r["proj"], r["binning_after"], r["out_img"], dl)
    grads, refine = oracle.vjp_dense(cam, cfg, sp.transforms, sp.sh, sp.raw_opac, r["proj"]["compact_from_global"], vc)
    b1, b2, inv1, inv2 = ops.adam_coefficients(time_step)
    n = sp.n
    width = grads.shape[1]
    lr_t = np.float32([1e-3] * 3 + [2e-3] * 4 + [5e-3] * 3)
    t = oracle.adam_q8(sp.transforms, grads, width, 0, 10, *mom["t"], lr_t, 1.0, b1, b2, inv1, inv2, 1e-15, 1)[0]
    lr_sh = np.float32([2e-3] * 3 + [2e-4] * 45)
    s = oracle.adam_q8(sp.sh.reshape(n, -1), grads, width, 10, 48, *mom["sh"], lr_sh, 1.0, b1, b2, inv1, inv2, 1e-15,
                       2)[0]
    o = oracle.adam_q8(sp.raw_opac, grads, width, width - 1, 1, *mom["o"], np.float32([0.012]), 1.0, b1, b2, inv1,
                       inv2, 1e-15, 3)[0]
    oracle.noise_means(t.reshape(n, 10), r["proj"]["opacities"], r["visible"], 1e-7, 1e-3, 5)
    return lo["loss"], s, o


def _q8_zero(count):
    blocks = (count + 255) // 256
    return [np.full(count, 128, np.uint8), np.zeros(count, np.uint8), np.zeros(blocks, np.float32),
            np.zeros(blocks, np.float32)]


def cpu_baseline(sp, tgt, cams, views, steps=1, warmup=0, gt=None):
    import oracle
    from vauss_b200 import scenes
    # all host cores, whatever OMP_NUM_THREADS a launcher set for this process
    cores = oracle.set_num_threads(os.cpu_count() or 1)
    cam = cams[views[0]]
    cfg = oracle.make_cfg(3, mip=True)
    if gt is None:
        gt = scenes.pack_rgba8(np.clip(oracle.render_forward(cam, cfg, tgt)["out_img"][..., :3], 0, 1))
    n = sp.n
    mom = {"t": _q8_zero(n * 10), "sh": _q8_zero(n * 48), "o": _q8_zero(n)}
    for k in range(warmup):
        oracle_step(sp, cam, gt, mom, k + 1)
    t0 = time.perf_counter()
    for k in range(steps):
        oracle_step(sp, cam, gt, mom, warmup + k + 1)
    dt = (time.perf_counter() - t0) / steps
    return {"value": round(1.0 / dt, 5), "unit": "iters/s", "cores": cores, "kind": "port",
            "sample": f"{steps} full config-2 step(s) of the C++ oracle (OpenMP), after {warmup} warm-up"}


def run_reference(args):
    """The reference arm: the reference's algorithm for this path on the host
    cores.  The reference itself (Rust/CubeCL/wgpu) cannot be built here, so
    this times the C++ oracle that restates it (oracle/splat_oracle.cpp)."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    sp, tgt, cams = make_workload(args.splats)
    views = list(range(N_TARGETS))
    steps = max(1, min(args.steps, 2))
    warm = min(args.warmup, 1)
    cpu = cpu_baseline(sp, tgt, cams, views, steps=steps, warmup=warm)
    cpu["sample"] = (f"{steps} timed full config-2 step(s) (after {warm} warm-up) of the C++ oracle restating the "
                     f"reference kernels; the Rust/CubeCL reference cannot be built in this image")
    out = {"metric": METRIC, "value": cpu["value"], "unit": "iters/s", "n_gpus": world, "steps": steps,
           "warmup": warm, "ms_per_step": round(1e3 / cpu["value"], 2), "higher_is_better": True, "scaling": "weak",
           "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
           "config": {"workload": "config 2: 3M SH-3 splats, 1600x1060, 1 view/step, L1+0.2 D-SSIM, 8-bit m+v Adam",
                      "splats": args.splats},
           "cpu_baseline": cpu,
           "e2e": {"value": cpu["value"], "unit": "iters/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


def run_sort_stress(args):
    """Benchmark configuration 4 (sort/overlap stress): 10M splats with large
    footprints (log-scales N(-2.5, 0.5), opacity logits N(1, 1), config-2
    means and SH), one 3840x2160 view, fx = fy = 3000.  Times projection,
    binning (intersection emission, depth and tile radix sorts, tile ranges),
    the forward and the backward under an N(0, 1e-3) upstream gradient.  The
    metric is intersections per second through intersect + sort + ranges.
    One view: under torchrun only rank 0 runs (replicas only)."""
    import torch
    from vauss_b200 import ops, scenes
    from vauss_b200.camera import look_at
    from vauss_b200.trainer import Splats
    if int(os.environ.get("RANK", "0")) != 0:
        return
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    n = args.splats
    sp = scenes.random_splats(n, 4004, mean_lo=-5.0, mean_hi=5.0, log_scale_mu=-2.5, log_scale_sigma=0.5,
                              opac_mu=1.0, opac_sigma=1.0, sh_degree=3)
    cam = look_at((0.0, -3.0, 8.0), (0.0, 0.0, 0.0), 3840, 2160, 3000.0)
    splats = Splats.from_numpy(sp, dev)
    del sp
    frame = ops.Frame(ops.context(dev))
    cfg = ops.render_cfg(3, mip=True)
    img = torch.empty(cam.height, cam.width, 4, device=dev)
    vis = torch.empty(n, device=dev)
    v_out = torch.randn(cam.height, cam.width, 4, device=dev, generator=torch.Generator(device=dev).manual_seed(1)) * 1e-3
    vc = torch.empty(n, 10, device=dev)
    stream = torch.cuda.current_stream(dev)
    names = ("project", "bin", "raster_fwd", "raster_bwd")
    acc = {k: 0.0 for k in names}

    def step(timed):
        evs = [torch.cuda.Event(enable_timing=True)]
        evs[0].record(stream)

        def hook(name):
            e = torch.cuda.Event(enable_timing=True)
            e.record(stream)
            evs.append(e)
        out = ops.render_stages(cam, cfg, splats.transforms, splats.sh_coeffs, splats.raw_opacities, frame, img, vis,
                                hook=hook)
        ops.rasterize_bwd(out.frame, out.out_img, v_out, vc)
        hook("raster_bwd")
        torch.cuda.synchronize()
        if timed:
            for k, (e0, e1) in zip(names, zip(evs[:-1], evs[1:])):
                acc[k] += e0.elapsed_time(e1)

    for _ in range(args.warmup):
        step(False)
    gpu_uuid = str(torch.cuda.get_device_properties(dev).uuid)
    with ClockSampler(gpu_uuid if gpu_uuid.startswith("GPU-") else f"GPU-{gpu_uuid}") as clk:
        clk.mark("start")
        for _ in range(args.steps):
            step(True)
        clk.mark("stop")
    counts = frame.counts
    isect, visible = int(counts.num_intersections), int(counts.num_visible)
    ms = {k: acc[k] / args.steps for k in names}
    sort_ms = ms["project"] + ms["bin"]
    peak, which = peaks()
    bin_bytes = stage_bytes("bin", n, visible, isect, cam.width * cam.height, cam.num_tiles)
    out = {"metric": "sort stress: intersections/s through intersect + radix sort + tile ranges @10M large splats 3840x2160",
           "value": round(isect / (sort_ms / 1e3), 1), "unit": "intersections/s", "n_gpus": 1, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": round(sum(ms.values()), 3), "higher_is_better": True,
           "scaling": "replicas only", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
           "config": {"workload": "config 4: 10M SH-3 splats, log-scales N(-2.5,0.5), opacity logits N(1,1), one "
                                  "3840x2160 view, fx=fy=3000, project+bin+raster fwd+raster bwd (N(0,1e-3) upstream)",
                      "splats": n, "visible": visible, "intersections": isect,
                      "l2": "inputs larger than L2"},
           "stages": {k: {"ms": round(v, 3)} for k, v in ms.items()},
           "roofline": {"bound": "hbm", "kernel": "bin", "achieved": round(bin_bytes / (ms["bin"] / 1e3) / 1e9, 1),
                        "peak": peak, "unit": "GB/s", "frac": round(bin_bytes / (ms["bin"] / 1e3) / 1e9 / peak, 4),
                        "traffic": None, "peak_source": which},
           "clocks": clk.summary()}
    print(json.dumps(out), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    elif args.config == 4:
        run_sort_stress(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
