#!/usr/bin/env python
"""Benchmark of the Gaussian-splat training step (fwd + bwd + Adam).

Configurations are numbered as BASELINE.json's ``configs`` list (0-based):
configs[0] is the tiny CPU-runnable run (a test case, not a bench line).

Default workload, configs[2] ("full training iteration at scale"):
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

Before the timed region the K timed steps are run once untimed from the
same starting state, which is then restored: one-time costs of a first pass
through them (workspace growing to the counts those steps reach, first
launches of kernel variants) fall in the warm-up, and the timed pass repeats
the same work.  After the timed region the same run, from the state the timed
region started from: the end-to-end leg through the public API (``e2e``), per-stage device
times (``stages``), at N = 1 one GPU step and one CPU-oracle step compared
(``parity``; the oracle step is also ``cpu_baseline``), at N > 1 a checksum
of every rank's replica (``replicas_equal``) and one step through the
peer-memory exchange against one through an NCCL all-reduce
(``exchange_check``), and finally configs[3] as a companion leg
(``config3``: steps/s of the fixed 8-view global batch at this N).

--config 3 runs configs[3] as the main line: 6,000,000 splats (configs[2]
distributions) and a fixed global batch of 8 views of 1920x1080
(fx = fy = 1600) per step, split evenly over 1, 2, 4 or 8 GPUs (strong
scaling; value = global-batch steps/s).  Every GPU count, one included, runs
the peer-memory view-parallel trainer.

--config 1 runs configs[1], the single-view render forward + backward
microbench (1M splats, 1920x1080), with rooflines for both raster kernels.

--config 4 runs the sort/overlap stress of configs[4] (one GPU): 10,000,000
large splats, one 3840x2160 view; value = intersections/s through
intersect + radix sort + tile ranges.

--optimizer reference (configs[2], one GPU) steps the reference's optimizer
storage instead of the 8-bit m+v Adam.

--emulate-peers W (one GPU) times the view-parallel update of configs[2]
with W ranks emulated on one device (each rank's compact rows written from a
render of its own view, every shard updated in turn with all ranks' buffers
as peers): the sharded optimizer kernel's own cost, without NVLink, and a
one-GPU command under which it can be profiled.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference] [--config 1|2|3|4]
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
    p.add_argument("--splats", type=int, default=None, help="default: 1M (configs[1]), 3M (configs[2]), 6M (configs[3]), 10M (configs[4])")
    p.add_argument("--config", type=int, default=2, choices=[1, 2, 3, 4],
                   help="index into BASELINE.json configs (0-based)")
    p.add_argument("--optimizer", default="q8", choices=["q8", "reference"],
                   help="configs[2] on one GPU: the 8-bit m+v Adam, or the reference's optimizer storage")
    p.add_argument("--no-cpu-baseline", action="store_true", help="skip the oracle step (parity and CPU baseline)")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-check", action="store_true", help="N > 1: skip the peer vs all-reduce exchange check")
    p.add_argument("--no-config3", action="store_true", help="skip the configs[3] companion leg")
    p.add_argument("--emulate-peers", type=int, default=0, metavar="W",
                   help="time the sharded compact-row update of configs[2] with W ranks emulated on one GPU")
    p.add_argument("--rows", default="compact", choices=["compact", "dense"],
                   help="N > 1: gradient rows of the peer exchange with one view per rank (compact 64-byte rows "
                        "with the SH gradient rebuilt by the owner, or dense rows)")
    a = p.parse_args()
    if a.splats is None:
        a.splats = {1: 1_000_000, 2: N_SPLATS, 3: 6_000_000, 4: 10_000_000}[a.config]
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


# DRAM bytes (read + write) per launch of each stage's kernel at configs[2]
# (3M splats, ~1.74M visible, ~5.77M intersections, 1600x1060), from
# single-kernel ncu captures of smaller cases scaled by the units each kernel
# processes: raster kernels from configs[1] (3.60M intersections) scaled by
# intersections, projection and the Q8 optimizer from a 1M-splat configs[2]
# scene scaled by splats, the VJP rows by visible splats, the loss (same image
# size) as captured.  Below the algorithmic bytes for the raster kernels: L2
# (126 MB) serves a projected row to the neighbouring tiles that gather it.
# Only the dominant stage's figure goes into the bench line.
MEASURED_TRAFFIC_CONFIG2 = {"raster_bwd": 138.35e6 * 5.766 / 3.597, "raster_fwd": 56.15e6 * 5.766 / 3.597,
                            "project": 224.93e6 * 3.0, "loss": 60.63e6,
                            "optimizer": 744.49e6 * 3.0 + 245.23e6 * 1.744 / 0.5858}


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
    if name == "optimizer_reference":
        # per splat: transforms r+w 80, packed geometry/opacity moment words r+w 88, opacity r+w 8, f16 SH r+w
        # 192, int8 SH m r+w 96, SH m scales ~3, SH v r+w 8, compact map 4, refine + grad^2 writes 8, stats r+w 24;
        # per visible splat: v_combined 40, params gathered for the VJP 140, colour/direction row w+r 48
        return n * (80 + 88 + 8 + 192 + 96 + 3 + 8 + 4 + 8 + 24) + v * (40 + 140 + 48)
    return 0.0


def mixed_rel(got, want, floor_frac=1e-3):
    """Largest |got - want| / max(|want|, floor_frac * max|want|): the tests'
    mixed absolute/relative error, as one number."""
    got = np.asarray(got, dtype=np.float64).ravel()
    want = np.asarray(want, dtype=np.float64).ravel()
    if want.size == 0:
        return 0.0
    scale = max(floor_frac * float(np.abs(want).max()), 1e-30)
    return float((np.abs(got - want) / np.maximum(np.abs(want), scale)).max())


def count_over(got, want, rel=1e-4, floor_frac=1e-3):
    """Elements beyond the tests' mixed tolerance."""
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    scale = max(floor_frac * float(np.abs(want).max()) if want.size else 0.0, 1e-30)
    return int((np.abs(got - want) > rel * np.maximum(np.abs(want), scale)).sum())


def replica_checksum(splats):
    """Two order-sensitive int64 checksums per parameter tensor of this
    rank's replica (sum of the f32 bit patterns, and that sum weighted by the
    element index mod 65521)."""
    import torch
    out = []
    for x in (splats.transforms, splats.sh_coeffs, splats.raw_opacities):
        b = x.contiguous().view(-1).view(torch.int32).to(torch.int64)
        w = torch.arange(b.numel(), device=b.device, dtype=torch.int64) % 65521 + 1
        out += [int(b.sum().item()), int((b * w).sum().item())]
        del b, w
    return out


class Leg:
    """One benchmark workload on this rank: the splats, targets and trainer
    of configuration 2 (one view per GPU per step) or 3 (a fixed global batch
    of 8 views split over the GPUs), and the snapshot the timed region
    starts from."""

    def __init__(self, args, config, n_splats, world, rank, dev):
        import torch
        from vauss_b200 import ops, scenes
        from vauss_b200.trainer import Splats, SplatTrainer, TrainConfig
        from vauss_b200.view_parallel import ViewParallelTrainer
        self.args, self.config, self.world, self.rank, self.dev = args, config, world, rank, dev
        self.multiview = config == 3
        if self.multiview and 8 % world:
            raise SystemExit("configuration 3 splits its 8 views over 1, 2, 4 or 8 GPUs")
        sp, tgt, cams = make_workload(n_splats, config)
        self.sp, self.cams = sp, cams
        splats = Splats.from_numpy(sp, dev)
        tsplats = Splats.from_numpy(tgt, dev)
        del tgt
        cfg_t = ops.render_cfg(3, mip=True)
        if self.multiview:  # this rank's share of the fixed global batch
            per_rank = 8 // world
            self.views = [rank * per_rank + k for k in range(per_rank)]
        else:
            self.views = [(rank * N_TARGETS + k) % N_VIEWS for k in range(N_TARGETS)]
        self.targets = []
        for vi in self.views:
            out = ops.render(cams[vi], cfg_t, tsplats.transforms, tsplats.sh_coeffs, tsplats.raw_opacities)
            img = out.out_img[..., :3].clamp(0, 1).cpu().numpy()
            self.targets.append(torch.from_numpy(scenes.pack_rgba8(img).view(np.int32)).to(dev))
        del tsplats
        torch.cuda.synchronize()
        self.cfg = TrainConfig(optimizer=args.optimizer if not (world > 1 or self.multiview) else "q8")
        median_scale = float(np.median(np.exp(sp.transforms[:, 7:10])))
        self.kw = dict(scene_extent=8.0, median_scale=median_scale)
        self.peer = None
        if world > 1 or self.multiview:
            from vauss_b200.peer import PeerGroup, gather_bytes_nccl
            gather = (lambda b: gather_bytes_nccl(b, dev)) if world > 1 else (lambda b: [b])
            self.peer = PeerGroup(dev, world, rank, gather)
            self.trainer = ViewParallelTrainer(self.cfg, dev, peer=self.peer, compact_rows=args.rows == "compact",
                                               **self.kw)
            self.splats = self.trainer.adopt(splats)
            del splats
        else:
            self.trainer = SplatTrainer(self.cfg, dev, **self.kw)
            self.splats = splats

    def batches(self, k, loader=None):
        from vauss_b200.trainer import SceneBatch
        if self.multiview:
            return ([loader.next_batch() for _ in self.views] if loader else
                    [SceneBatch(self.targets[j], self.cams[self.views[j]], self.views[j])
                     for j in range(len(self.views))])
        vi = k % N_TARGETS
        return [loader.next_batch() if loader else SceneBatch(self.targets[vi], self.cams[self.views[vi]],
                                                                 self.views[vi])]

    def step(self, k, loader=None, hook=None):
        b = self.batches(k, loader)
        if self.world > 1 or self.multiview:
            return self.trainer.step_views(b, self.splats, hook=hook)
        # the reference optimizer hands back new splats (SH in f16 from its first step)
        self.splats, st = self.trainer.step(b[0], self.splats)
        return self.splats, st

    def barrier(self):
        import torch
        import torch.distributed as dist
        if self.world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def optim_tensors(self):
        o = self.trainer.optim
        if "t" in o:
            return [getattr(o[k], a) for k in ("t", "sh", "o") for a in ("m_codes", "v_codes", "m_scales",
                                                                           "v_scales")]
        return [o[k] for k in ("w_t", "w_o", "codes", "scales", "variance")]

    def snapshot(self):
        import copy
        s = self.splats
        tr = self.trainer
        self.snap = {"p": [x.clone() for x in (s.transforms, s.sh_coeffs, s.raw_opacities)],
                     "m": [x.clone() for x in self.optim_tensors()],
                     "time": tr.optim["time"], "step": tr.step_count,
                     "rng": copy.deepcopy(tr.rng.bit_generator.state)}

    def restore(self):
        import copy
        s = self.splats
        tr = self.trainer
        for dst, src in zip((s.transforms, s.sh_coeffs, s.raw_opacities), self.snap["p"]):
            dst.copy_(src)
        for dst, src in zip(self.optim_tensors(), self.snap["m"]):
            dst.copy_(src)
        tr.optim["time"], tr.step_count = self.snap["time"], self.snap["step"]
        tr.rng.bit_generator.state = copy.deepcopy(self.snap["rng"])
        self.barrier()

    def close(self):
        import torch
        import torch.distributed as dist
        if self.peer is None:
            return
        torch.cuda.synchronize(self.dev)
        if self.world > 1:
            dist.barrier()  # no rank's kernels touch peer buffers any more
        self.peer.check()
        self.peer.close()
        self.peer = None
        torch.cuda.synchronize(self.dev)
        if self.world > 1:
            dist.barrier()


def timed_run(leg, steps, warmup):
    """Warm-up, snapshot, then `steps` timed steps bracketed by a barrier and
    a synchronize; returns (max-over-ranks ms, launches per step, clocks,
    counts of the last warm-up step)."""
    import torch
    import torch.distributed as dist
    from vauss_b200 import ops
    counts = {}
    for k in range(warmup):
        _, st0 = leg.step(k)
        counts = {"visible": int(st0.num_visible), "intersections": int(st0.num_intersections)}
    leg.barrier()
    # The timed region starts from this state; the per-stage profile, the
    # end-to-end leg and the checks restart from it too, so that all of them
    # see the same workload (training moves the splats, and the raster work
    # grows with it).
    leg.snapshot()
    # The timed steps are rehearsed once, untimed, from the same state: the
    # one-time costs of a first pass through them (workspace growing to the
    # intersection counts those steps reach, first launches of kernel
    # variants) are warm-up, and the timed pass repeats the same work.
    for k in range(steps):
        leg.step(warmup + k)
    leg.restore()
    ctx = ops.context(leg.dev)
    launches0 = ctx.launch_count
    gpu_uuid = str(torch.cuda.get_device_properties(leg.dev).uuid)
    gpu_id = gpu_uuid if gpu_uuid.startswith("GPU-") else f"GPU-{gpu_uuid}"
    stream = torch.cuda.current_stream(leg.dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(gpu_id) as clk:
        leg.barrier()
        clk.mark("start")
        e0.record(stream)
        for k in range(steps):
            leg.step(warmup + k)
        e1.record(stream)
        leg.barrier()
        clk.mark("stop")
    ms = e0.elapsed_time(e1)
    launches = (ctx.launch_count - launches0) // max(steps, 1)
    t = torch.tensor([ms], dtype=torch.float64, device=leg.dev)
    if leg.world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item()), launches, clk.summary(), counts


def e2e_run(leg, steps, warmup):
    """The same steps through the public API with the ground truth staged from
    host memory each step (SceneLoader) and the loss read back."""
    import torch
    import torch.distributed as dist
    from vauss_b200 import dataset
    rgb = [tg.cpu().numpy().view(np.uint8).reshape(tg.shape[0], tg.shape[1], 4)[..., :3].copy()
           for tg in leg.targets]
    loader = dataset.SceneLoader(
        dataset.Scene([dataset.SceneView(img, leg.cams[vi]) for img, vi in zip(rgb, leg.views)]), seed=leg.rank,
        config=dataset.LoadDatasetConfig(max_scene_batch_cache_size=0), device=leg.dev,
        hold=len(leg.views) if leg.multiview else 1)
    loss_host = torch.empty((), dtype=torch.float32).pin_memory()
    for k in range(warmup):  # untimed: first use of the host-input path
        _, st = leg.step(k, loader=loader)
        loss_host.copy_(st.loss, non_blocking=True)
    leg.restore()
    stream = torch.cuda.current_stream(leg.dev)
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    h2d0 = loader.h2d_bytes_total
    f0.record(stream)
    for k in range(steps):
        _, st = leg.step(k, loader=loader)
        loss_host.copy_(st.loss, non_blocking=True)
    f1.record(stream)
    leg.barrier()
    ems = f0.elapsed_time(f1)
    h2d_total = loader.h2d_bytes_total - h2d0
    loader.close()
    te = torch.tensor([ems], dtype=torch.float64, device=leg.dev)
    if leg.world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    per = 1 if leg.multiview else leg.world
    return {"value": per * steps / (float(te.item()) / 1e3), "unit": "steps/s" if leg.multiview else "iters/s",
            "h2d_bytes_per_step": int(round(h2d_total / max(steps, 1))), "d2h_bytes_per_step": 4,
            "feed": "SceneLoader (vs_feed): RGB8 views, pinned ring of 4, packed on the GPU, no cache",
            "api": ("ViewParallelTrainer.step_views (vs_render_forward, vs_loss, vs_rasterize_backward, "
                    "vs_vjp_compact with one view per rank or vs_vjp_dense, vs_peer_barrier, vs_adam_q8_peer)"
                    if leg.world > 1 or leg.multiview else
                    "SplatTrainer.step (vs_render_forward, vs_loss, vs_rasterize_backward, vs_step_q8)")}


def profile_stages_views(leg, reps=5):
    """Per-stage device times of the view-parallel step (CUDA events on the
    launching stream): the median over `reps` steps per rank, then the maximum
    over ranks for every stage."""
    import torch
    import torch.distributed as dist
    stream = torch.cuda.current_stream(leg.dev)
    acc = {}
    for r in range(reps):
        evs = [("start", torch.cuda.Event(enable_timing=True))]
        evs[0][1].record(stream)

        def hook(name):
            e = torch.cuda.Event(enable_timing=True)
            e.record(stream)
            evs.append((name, e))
        leg.step(r, hook=hook)
        torch.cuda.synchronize()
        per = {}
        for (_, ea), (b, eb) in zip(evs[:-1], evs[1:]):
            per[b] = per.get(b, 0.0) + ea.elapsed_time(eb)  # several views: summed per stage
        for b, v in per.items():
            acc.setdefault(b, []).append(v)
    names = list(acc)
    med = torch.tensor([statistics.median(acc[k]) for k in names], dtype=torch.float64, device=leg.dev)
    if leg.world > 1:
        dist.all_reduce(med, op=dist.ReduceOp.MAX)
    return {k: {"ms": round(float(v), 4)} for k, v in zip(names, med.tolist())}


def replicas_check(leg):
    """True when every rank's replica has the same checksums as rank 0's."""
    import torch
    import torch.distributed as dist
    mine = torch.tensor(replica_checksum(leg.splats), dtype=torch.int64, device=leg.dev)
    allc = [torch.empty_like(mine) for _ in range(leg.world)]
    dist.all_gather(allc, mine)
    return all(torch.equal(allc[0], c) for c in allc[1:])


def exchange_check(leg):
    """One step from the timed-region snapshot through the peer-memory
    exchange and one through an NCCL all-reduce of the dense rows followed by
    the replicated Adam, both from zero moments; returns the largest
    differences over ranks between the two parameter sets."""
    import copy
    import torch
    import torch.distributed as dist
    from vauss_b200 import ops
    from vauss_b200.trainer import Splats
    from vauss_b200.view_parallel import ViewParallelTrainer
    from vauss_b200.trainer import SceneBatch
    leg.restore()
    tr = leg.trainer
    saved = tr.optim
    nc = leg.splats.sh_coeffs.shape[1]
    m = tr.shard[1] - tr.shard[0]
    tr.optim = dict(t=ops.Q8Moments(m * 10, leg.dev), sh=ops.Q8Moments(m * nc * 3, leg.dev),
                    o=ops.Q8Moments(m, leg.dev), time=saved["time"])
    ref = ViewParallelTrainer(leg.cfg, leg.dev, **leg.kw)  # all-reduce exchange (NCCL)
    p0 = [x.clone() for x in (leg.splats.transforms, leg.splats.sh_coeffs, leg.splats.raw_opacities)]
    other = Splats(*[x.clone() for x in p0])
    ref._init_state(other)
    ref.optim["time"], ref.step_count = saved["time"], tr.step_count
    ref.rng.bit_generator.state = copy.deepcopy(tr.rng.bit_generator.state)
    b = leg.batches(0)
    tr.step_views(b, leg.splats)
    ref.step_views(b, other)
    torch.cuda.synchronize()
    got = [x.cpu().numpy() for x in (leg.splats.transforms, leg.splats.sh_coeffs, leg.splats.raw_opacities)]
    want = [x.cpu().numpy() for x in (other.transforms, other.sh_coeffs, other.raw_opacities)]
    base = [x.cpu().numpy() for x in p0]
    prm = max(mixed_rel(g, w) for g, w in zip(got, want))
    upd = max(float(np.abs((g - b0) - (w - b0)).max()) / max(float(np.abs(w - b0).max()), 1e-30)
              for g, w, b0 in zip(got, want, base))
    # values whose update differs by more than 1e-3 of the largest update
    over = sum(int((np.abs((g - b0) - (w - b0)) > 1e-3 * max(float(np.abs(w - b0).max()), 1e-30)).sum())
               for g, w, b0 in zip(got, want, base))
    total = sum(g.size for g in got)
    t = torch.tensor([prm, upd, over / total], dtype=torch.float64, device=leg.dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    tr.optim = saved
    del ref, other
    torch.cuda.empty_cache()
    leg.restore()
    return {"params_max_rel": float(t[0]), "update_max_rel": float(t[1]), "update_frac_over_1e-3": float(t[2]),
            "rows": "compact" if getattr(tr, "compact_rows", False) and len(b) == 1 else "dense",
            "what": "one step from the timed-region parameters and zero moments through the peer-memory exchange "
                    "and through an NCCL all-reduce + replicated Adam; mixed rel over all parameters, the "
                    "largest update difference over the largest update, and the fraction of values whose update "
                    "differs by more than 1e-3 of the largest (from zero moments Adam's step is about lr * sign(g), "
                    "so a near-zero gradient whose rounding differs between the two renders moves one update by "
                    "up to 2 lr)"}


def parity_leg(leg):
    """One training step on the GPU and one of the CPU oracle, both from the
    timed-region snapshot (parameters and 8-bit moments) on the first view:
    integer outputs compared for equality, floating-point ones as the tests'
    mixed error.  The oracle step is also the CPU baseline's timed sample."""
    import oracle
    import torch
    from vauss_b200 import ops, scenes
    leg.restore()
    tr = leg.trainer
    c = tr.config
    dev = leg.dev
    s = leg.splats
    n = s.num_splats
    host = [x.cpu().numpy() for x in (s.transforms, s.sh_coeffs, s.raw_opacities)]
    o = tr.optim
    mom_h = {k: [getattr(o[k], a).cpu().numpy() for a in ("m_codes", "v_codes", "m_scales", "v_scales")]
             for k in ("t", "sh", "o")}
    t_step = o["time"] + 1
    lr_t = np.asarray(tr.transforms_lr(), np.float32)
    lr_dc, lr_rest, lr_o = c.lr_coeffs_dc, c.lr_coeffs_dc / c.lr_coeffs_sh_scale, c.lr_opac
    noise = (1e-7, 1e-3, 4321)
    cam, gt = leg.cams[leg.views[0]], leg.targets[0]
    # ---- GPU: the trainer's kernels with the same arguments ----
    t, sh, op = (x.clone() for x in (s.transforms, s.sh_coeffs, s.raw_opacities))
    moms = []
    for k in ("t", "sh", "o"):
        q = ops.Q8Moments.__new__(ops.Q8Moments)
        q.m_codes, q.v_codes, q.m_scales, q.v_scales = (getattr(o[k], a).clone() for a in
                                                        ("m_codes", "v_codes", "m_scales", "v_scales"))
        moms.append(q)
    cfg = ops.render_cfg(3, mip=True)
    frame = ops.Frame(ops.context(dev))
    out = ops.render(cam, cfg, t, sh, op, frame=frame)
    loss = ops.image_loss(out.out_img, gt, c.l1_weight, c.ssim_loss_weight)
    vc = ops.rasterize_bwd(out.frame, out.out_img, loss.dl_dpred)
    vc_h = vc.cpu().numpy()
    q8 = ops.q8_cfg(t_step, lr_t, lr_dc, lr_rest, lr_o, eps=c.adam_epsilon, noise_scale=noise[0],
                    noise_limit=noise[1], noise_seed=noise[2])
    ops.step_q8(out.frame, cfg, t, sh, op, vc, *moms, q8, visible=out.visible)
    torch.cuda.synchronize()
    g = {"img": out.out_img.cpu().numpy(), "visible": out.visible.cpu().numpy(), "loss": float(loss.loss.item()),
         "tile": frame.field("isect_tile").cpu().numpy().view(np.uint32),
         "cid": frame.field("isect_compact").cpu().numpy().view(np.uint32),
         "ranges": frame.field("tile_ranges").cpu().numpy().view(np.uint32),
         "used": frame.field("tile_used_end").cpu().numpy().view(np.uint32),
         "params": [x.cpu().numpy() for x in (t, sh, op)],
         "codes": [getattr(q, a).cpu().numpy() for q in moms for a in ("m_codes", "v_codes")]}
    nv, ni = out.num_visible, out.num_intersections
    del t, sh, op, moms, out, loss, vc, frame
    torch.cuda.empty_cache()
    # ---- CPU oracle ----
    cores = oracle.set_num_threads(os.cpu_count() or 1)
    gt_h = gt.cpu().numpy().view(np.uint32)
    t0 = time.perf_counter()
    cfg_o = oracle.make_cfg(3, mip=True)
    sset = scenes.SplatSet(*host)
    ref = oracle.render_forward(cam, cfg_o, sset)
    lo = oracle.loss_fwd(ref["out_img"], gt_h, c.l1_weight, c.ssim_loss_weight)
    dl = oracle.loss_bwd(ref["out_img"], gt_h, lo["coeffs"], c.l1_weight, c.ssim_loss_weight)
    vc_ref = oracle.raster_bwd(cam, (0.0, 0.0, 0.0), ref["proj"], ref["binning_after"], ref["out_img"], dl)
    grads, _ = oracle.vjp_dense(cam, cfg_o, host[0], host[1], host[2], ref["proj"]["compact_from_global"], vc_ref)
    b1, b2, inv1, inv2 = ops.adam_coefficients(t_step)
    width = grads.shape[1]
    eps = c.adam_epsilon
    rt = oracle.adam_q8(host[0], grads, width, 0, 10, *[x.copy() for x in mom_h["t"]], lr_t, 1.0, b1, b2, inv1,
                        inv2, eps, t_step ^ (10 << 24))
    lr_sh = np.float32([lr_dc] * 3 + [lr_rest] * 45)
    rs = oracle.adam_q8(host[1].reshape(n, -1), grads, width, 10, 48, *[x.copy() for x in mom_h["sh"]], lr_sh, 1.0,
                        b1, b2, inv1, inv2, eps, t_step ^ (48 << 24))
    ro = oracle.adam_q8(host[2], grads, width, width - 1, 1, *[x.copy() for x in mom_h["o"]], np.float32([lr_o]),
                        1.0, b1, b2, inv1, inv2, eps, t_step ^ (1 << 24))
    tr_new = oracle.noise_means(rt[0].reshape(n, 10), ref["proj"]["opacities"], ref["visible"], *noise)
    dt = time.perf_counter() - t0

    def oracle_update(vcomb):
        gr, _ = oracle.vjp_dense(cam, cfg_o, host[0], host[1], host[2], ref["proj"]["compact_from_global"], vcomb)
        a = oracle.adam_q8(host[0], gr, width, 0, 10, *[x.copy() for x in mom_h["t"]], lr_t, 1.0, b1, b2, inv1,
                           inv2, eps, t_step ^ (10 << 24))
        b = oracle.adam_q8(host[1].reshape(n, -1), gr, width, 10, 48, *[x.copy() for x in mom_h["sh"]], lr_sh, 1.0,
                           b1, b2, inv1, inv2, eps, t_step ^ (48 << 24))
        c_ = oracle.adam_q8(host[2], gr, width, width - 1, 1, *[x.copy() for x in mom_h["o"]],
                            np.float32([lr_o]), 1.0, b1, b2, inv1, inv2, eps, t_step ^ (1 << 24))
        tn = oracle.noise_means(a[0].reshape(n, 10), ref["proj"]["opacities"], ref["visible"], *noise)
        return [tn, b[0].reshape(host[1].shape), c_[0]], [a[1], a[2], b[1], b[2], c_[1], c_[2]]

    want = [tr_new, rs[0].reshape(host[1].shape), ro[0]]
    prm = max(mixed_rel(a, b) for a, b in zip(g["params"], want))
    within = sum(b.size - count_over(a, b) for a, b in zip(g["params"], want)) / sum(b.size for b in want)
    upd = max(float(np.abs(a - b).max()) / max(float(np.abs(b - h).max()), 1e-30)
              for a, b, h in zip(g["params"], want, host))
    codes_want = [rt[1], rt[2], rs[1], rs[2], ro[1], ro[2]]
    codes_eq = sum(int((a == b).sum()) for a, b in zip(g["codes"], codes_want)) / sum(b.size for b in codes_want)
    # the optimizer alone: the oracle's VJP + Adam fed the GPU's own v_combined
    p_same, c_same = oracle_update(vc_h)
    step_bits = all(np.array_equal(np.ascontiguousarray(a).view(np.uint32), np.ascontiguousarray(b).view(np.uint32))
                    for a, b in zip(g["params"], p_same)) and \
        all(np.array_equal(a, b) for a, b in zip(g["codes"], c_same))
    parity = {
        "counts_equal": bool(nv == ref["proj"]["num_visible"] and ni == ref["proj"]["num_isect"]),
        "keys_equal": bool(np.array_equal(g["tile"], ref["binning"]["tile_ids"]) and
                           np.array_equal(g["cid"], ref["binning"]["isect_compact"])),
        "ranges_equal": bool(np.array_equal(g["ranges"].reshape(-1, 2), ref["tile_offsets_pre"]) and
                             np.array_equal(g["used"], ref["tile_offsets"][:, 1])),
        "img_max_rel": mixed_rel(g["img"], ref["out_img"]),
        "img_px_over_1e-4": count_over(g["img"], ref["out_img"]),
        "visible_equal": bool(np.array_equal(g["visible"], ref["visible"])),
        "loss_rel": abs(g["loss"] - lo["loss"]) / max(abs(lo["loss"]), 1e-30),
        "vcomb_max_rel": mixed_rel(vc_h, vc_ref),
        "params_max_rel": prm, "params_frac_within_1e-4": round(within, 8), "update_max_rel": upd,
        "codes_equal_frac": round(codes_eq, 7), "optimizer_bits_equal_given_vcomb": bool(step_bits),
        "what": ("one step from the timed-region snapshot on the first view, GPU vs the C++ oracle; floats as "
                 "max |got-want|/max(|want|, 1e-3 max|want|); params_* and update_max_rel (largest update "
                 "difference over the largest update) end to end, where v_combined differs by float-atomic "
                 "order and Adam's normalised step turns a near-zero gradient's rounding into an O(lr) update "
                 "difference; optimizer_bits_equal_given_vcomb: the GPU's VJP + 8-bit Adam against the "
                 "oracle's fed the GPU's v_combined, every parameter and code bit for bit")}
    cpu = {"value": round(1.0 / dt, 5), "unit": "iters/s", "cores": cores, "kind": "port",
           "sample": "1 full configs[2] step of the C++ oracle (OpenMP) from the timed-region snapshot, the same "
                     "step the parity check compares"}
    leg.restore()
    return parity, cpu


def config_line(leg, value, ms_max, steps, warmup, launches, clocks, counts):
    world, multiview = leg.world, leg.multiview
    if multiview:
        workload = dict(workload="configs[3]: 6M SH-3 splats, global batch of 8 views of 1920x1080 split over "
                                 f"the GPUs ({len(leg.views)} per GPU), L1+0.2 D-SSIM, 8-bit m+v Adam (block 256)",
                        splats=leg.splats.num_splats, width=1920, height=1080, views_per_step=8)
    else:
        workload = dict(workload="configs[2]: 3M SH-3 splats, 1600x1060, 1 view/step/GPU, L1+0.2 D-SSIM, "
                                 + ("8-bit m+v Adam (block 256)" if leg.cfg.optimizer == "q8" else
                                    "reference optimizer storage (packed 16/16 geometry moments, f16 SH, "
                                    "int8 SH m in 128-value blocks)"),
                        splats=leg.splats.num_splats, width=1600, height=1060, views_per_step=world)
    return {"metric": ("view-parallel steps/s @6M splats, 8 views of 1920×1080 per step" if multiview else METRIC),
            "value": round(value, 3), "unit": "steps/s" if multiview else "iters/s", "n_gpus": world,
            "steps": steps, "warmup": warmup, "ms_per_step": round(ms_max / steps, 4),
            "higher_is_better": True, "scaling": "strong" if multiview else "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": {**workload, "optimizer": leg.cfg.optimizer,
                       "parallelism": (f"view-parallel x{world}: "
                                       + ("64-byte compact gradient rows per view" if leg.args.rows == "compact"
                                          else "dense gradient rows per rank")
                                       + " read over NVLink peer memory by a sharded fused Adam that stores to "
                                         "every replica" if world > 1 or multiview else "single GPU"),
                       "l2": ("inputs larger than L2 (params + moments ~%.1f GB)"
                              % (leg.splats.num_splats * (236 + 122) / 1e9)),
                       "timing": ("W warm-up steps; the K timed steps once untimed from the timed region's "
                                  "starting state (restored after); then the K steps timed"), **counts},
            "gpu_launches": int(launches), "clocks": clocks}


def run_ours(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        from datetime import timedelta
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device(f"cuda:{local}"))
    dev = torch.device(f"cuda:{local}")
    torch.cuda.set_device(dev)

    leg = Leg(args, args.config, args.splats, world, rank, dev)
    ms_max, launches, clocks, counts = timed_run(leg, args.steps, args.warmup)
    value = (1 if leg.multiview else world) * args.steps / (ms_max / 1e3)
    out = config_line(leg, value, ms_max, args.steps, args.warmup, launches, clocks, counts)
    if not args.no_e2e:
        e2e = e2e_run(leg, args.steps, args.warmup)
        out["e2e"] = {k: (round(v, 3) if isinstance(v, float) else v) for k, v in e2e.items()}
    if world > 1:
        out["replicas_equal"] = replicas_check(leg)  # after every timed and end-to-end step

    # ---- per-stage device times (CUDA events on the launching stream) ----
    if world == 1 and not leg.multiview:
        leg.restore()
        stages = profile_stages(leg.trainer, leg.splats, leg.targets, leg.cams, leg.views, dev, reps=5)
        peak, which = peaks()
        n, v, i = leg.splats.num_splats, stages.pop("_v"), stages.pop("_i")
        cam0 = leg.cams[leg.views[0]]
        p, tcount = cam0.width * cam0.height, cam0.num_tiles
        for name, d in stages.items():
            b = stage_bytes(name if not (name == "optimizer" and leg.cfg.optimizer == "reference")
                            else "optimizer_reference", n, v, i, p, tcount)
            d["gbs"] = b / (d["ms"] / 1e3) / 1e9
            d["alg_bytes"] = b
        dom = max(stages, key=lambda k: stages[k]["ms"])
        ach = stages[dom]["gbs"]
        out["roofline"] = {"bound": "hbm", "kernel": dom, "achieved": round(ach, 1), "peak": peak, "unit": "GB/s",
                           "frac": round(ach / peak, 4),
                           "traffic": (MEASURED_TRAFFIC_CONFIG2.get(dom) if n == N_SPLATS else None),
                           "peak_source": which,
                           "note": "raster stages are FP32-issue bound; see profiles/ for issue utilisation"}
        out["stages"] = {k: {"ms": round(d["ms"], 4), "gbs": round(d["gbs"], 1), "frac": round(d["gbs"] / peak, 4)}
                         for k, d in stages.items()}
    else:
        leg.restore()
        out["stages"] = profile_stages_views(leg)
        if world > 1:
            out["stages_note"] = "per stage the median of 5 steps on each rank, then the maximum over ranks"
    if world > 1 and not args.no_check:
        out["exchange_check"] = exchange_check(leg)
    if rank == 0 and world == 1 and not leg.multiview and not args.no_cpu_baseline and \
            leg.cfg.optimizer == "q8":
        parity, cpu = parity_leg(leg)
        out["parity"] = parity
        out["cpu_baseline"] = cpu
    leg.close()
    del leg
    torch.cuda.empty_cache()

    # ---- configuration 3 (strong scaling) as a companion of the scaling run ----
    if args.config == 2 and not args.no_config3 and args.optimizer == "q8":
        c3 = Leg(args, 3, 6_000_000, world, rank, dev)
        k3, w3 = max(3, min(args.steps, 10)), 3
        ms3, _, clk3, cnt3 = timed_run(c3, k3, w3)
        rec = {"steps_per_s": round(k3 / (ms3 / 1e3), 3), "ms_per_step": round(ms3 / k3, 3), "n_gpus": world,
               "steps": k3, "warmup": w3, "splats": c3.splats.num_splats, "views_per_step": 8,
               "views_per_gpu": len(c3.views), "scaling": "strong", "clocks": clk3, **cnt3}
        if not args.no_e2e:
            e = e2e_run(c3, k3, w3)
            rec["e2e"] = {"value": round(e["value"], 3), "unit": e["unit"],
                          "h2d_bytes_per_step": e["h2d_bytes_per_step"], "d2h_bytes_per_step": 4}
        if world > 1:
            rec["replicas_equal"] = replicas_check(c3)
        c3.close()
        out["config3"] = rec
    if rank == 0:
        print(json.dumps(out), flush=True)
    if world > 1:
        dist.barrier()
        torch.cuda.synchronize(dev)
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
        cfg = ops.render_cfg(3, mip=True, sh_half=splats.sh_coeffs.dtype == torch.float16,
                             background=(0.0, 0.0, 0.0))
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
        if c.optimizer == "q8":
            q8 = ops.q8_cfg(o["time"], trainer.transforms_lr(), c.lr_coeffs_dc,
                            c.lr_coeffs_dc / c.lr_coeffs_sh_scale, c.lr_opac, eps=c.adam_epsilon, noise_scale=1e-7,
                            noise_limit=1e-3, noise_seed=r)
            rec = trainer.record
            ops.step_q8(out.frame, cfg, splats.transforms, splats.sh_coeffs, splats.raw_opacities, vc, o["t"],
                        o["sh"], o["o"], q8, visible=out.visible, refine_norm=rec.refine_norm,
                        vis_count=rec.vis_count, max_screen=rec.max_screen)
        else:  # the reference optimizer storage: fused project_update + SH step + stats + noise
            cfg = ops.render_cfg(3, mip=True, sh_half=True, background=(0.0, 0.0, 0.0))
            trainer._reference_optimizer_step(out, cfg, splats, vc, trainer.transforms_lr(), 0.0, o["time"], 1e-7, r)
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
            "sample": f"{steps} full configs[2] step(s) of the C++ oracle (OpenMP), after {warmup} warm-up"}


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
    cpu["sample"] = (f"{steps} timed full configs[2] step(s) (after {warm} warm-up) of the C++ oracle restating the "
                     f"reference kernels; the Rust/CubeCL reference cannot be built in this image")
    out = {"metric": METRIC, "value": cpu["value"], "unit": "iters/s", "n_gpus": world, "steps": steps,
           "warmup": warm, "ms_per_step": round(1e3 / cpu["value"], 2), "higher_is_better": True, "scaling": "weak",
           "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
           "config": {"workload": "configs[2]: 3M SH-3 splats, 1600x1060, 1 view/step/GPU, L1+0.2 D-SSIM, 8-bit m+v Adam (block 256)",
                      "splats": args.splats},
           "cpu_baseline": cpu,
           "e2e": {"value": cpu["value"], "unit": "iters/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


def run_peer_emulation(args):
    """``--emulate-peers W``: the view-parallel update of configs[2] with W
    ranks emulated on one GPU, so that the sharded optimizer kernel can be
    timed and profiled on one device.  Every emulated rank renders its own
    view, runs the loss and the rasterizer backward and writes its compact
    rows, view mask and camera into buffers of its own; then each rank's
    shard is updated (vs_adam_q8_peer, row_format 1) with all ranks' buffers
    as its peers, one launch after another, and the update of every shard is
    timed with CUDA events over K steps.  No NVLink is crossed: the figure is
    the kernel's own cost, the peer reads and replica stores landing in this
    GPU's memory."""
    import torch
    from vauss_b200 import _native as N, ops, scenes
    from vauss_b200.view_parallel import ViewParallelTrainer
    dev = torch.device("cuda", 0)
    world = args.emulate_peers
    if not 1 <= world <= N.PEER_MAX:
        raise SystemExit(f"--emulate-peers takes 1..{N.PEER_MAX} ranks")
    sp, tgt, cams = make_workload(args.splats, 2)
    n, deg, nc = sp.n, 3, 16
    params = [torch.from_numpy(np.ascontiguousarray(x)).to(dev) for x in (sp.transforms, sp.sh, sp.raw_opac)]
    tsp = [torch.from_numpy(np.ascontiguousarray(x)).to(dev) for x in (tgt.transforms, tgt.sh, tgt.raw_opac)]
    cfg = ops.render_cfg(deg, mip=True)
    rows = [torch.zeros(n * N.COMPACT_ROW, device=dev) for _ in range(world)]
    vis = [torch.zeros(n, device=dev) for _ in range(world)]
    refine = torch.zeros(n, device=dev)
    camb = [torch.zeros(4, device=dev) for _ in range(world)]
    masks = [torch.zeros(n, dtype=torch.int32, device=dev) for _ in range(world)]
    visible, isect = 0, 0
    for r in range(world):
        cam = cams[(r * N_TARGETS) % N_VIEWS]
        gt_img = ops.render(cam, cfg, *tsp).out_img[..., :3].clamp(0, 1).cpu().numpy()
        gt = torch.from_numpy(scenes.pack_rgba8(gt_img).view(np.int32)).to(dev)
        out = ops.render(cam, cfg, *params)
        loss = ops.image_loss(out.out_img, gt, 0.8, 0.2)
        vc = ops.rasterize_bwd(out.frame, out.out_img, loss.dl_dpred)
        ops.vjp_compact(out.frame, cfg, *params, vc, rows[r], refine, camb[r], masks[r], 0, visible=out.visible,
                        vis_accum=vis[r])
        visible += out.num_visible
        isect += out.num_intersections
    del tsp
    reps = [[x.clone() for x in params] for _ in range(world)]
    ps = N.PeerSet()
    ps.world, ps.row_format, ps.views = world, 1, 1
    for r in range(world):
        ps.grads[r], ps.vis[r], ps.cams[r], ps.view_masks[r] = (rows[r].data_ptr(), vis[r].data_ptr(),
                                                                camb[r].data_ptr(), masks[r].data_ptr())
        ps.transforms[r], ps.sh_coeffs[r], ps.raw_opacities[r] = (x.data_ptr() for x in reps[r])
    shards = [ViewParallelTrainer.shard_of(n, world, r) for r in range(world)]
    moms = [dict(t=ops.Q8Moments((e - b) * 10, dev), sh=ops.Q8Moments((e - b) * nc * 3, dev),
                 o=ops.Q8Moments(e - b, dev)) for b, e in shards]
    lr_t = np.float32([1.6e-4] * 3 + [1e-3] * 4 + [5e-3] * 3)
    ctx = ops.context(dev)

    def update_all(step, ev=None):
        q8 = ops.q8_cfg(step + 1, lr_t, 2.5e-3, 1.25e-4, 2.5e-2)
        for r, (b, e) in enumerate(shards):
            ps.rank = r
            if ev is not None:
                ev[r][0].record()
            ops.adam_q8_peer(deg, n, b, e, ps, moms[r]["t"], moms[r]["sh"], moms[r]["o"], q8, device=dev)
            if ev is not None:
                ev[r][1].record()

    for k in range(args.warmup):
        update_all(k)
    ms = [0.0] * world
    for k in range(args.steps):
        ev = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(world)]
        update_all(args.warmup + k, ev)
        torch.cuda.synchronize()
        for r in range(world):
            ms[r] += ev[r][0].elapsed_time(ev[r][1])
    if ctx.lib.vs_ctx_check(ctx.h) != 0:
        raise SystemExit(ctx.lib.vs_ctx_last_error(ctx.h).decode())
    per = [m / args.steps for m in ms]
    out = {"metric": "sharded 8-bit-moment update from compact rows, ranks emulated on one GPU",
           "value": round(sum(per), 4), "unit": "ms per step (all shards)", "n_gpus": 1, "steps": args.steps,
           "warmup": args.warmup, "higher_is_better": False, "emulated_ranks": world,
           "ms_per_shard": [round(x, 4) for x in per], "splats": n, "visible_per_view": round(visible / world),
           "intersections_per_view": round(isect / world), "data": "synthetic",
           "config": {"workload": f"configs[2] step's update, {world} ranks emulated on one GPU (no NVLink)",
                      "kernel": "q8_kernel<3> (vs_adam_q8_peer, row_format 1)"}}
    print(json.dumps(out), flush=True)


def run_microbench(args):
    """BASELINE.json configs[1], the single-view render forward + backward
    microbench: 1M SH-3 splats (means U[-3,3]^3, log-scales N(-4.5, 0.6),
    opacity logits N(0, 1.5)), one 1920x1080 pinhole view at distance 6,
    fx = fy = 1600, upstream image gradient N(0, 1e-3) per pixel and channel.
    One step = projection, binning, rasterize forward, rasterize backward;
    value = steps/s.  Both raster kernels get a roofline entry, and the CPU
    oracle's forward + backward of the same view is the parity check and the
    CPU baseline.  One view: under torchrun only rank 0 runs."""
    import torch
    import oracle
    from vauss_b200 import ops, scenes
    from vauss_b200.trainer import Splats
    if int(os.environ.get("RANK", "0")) != 0:
        return
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    sp, cam = scenes.config_microbench(n=args.splats)
    n = sp.n
    splats = Splats.from_numpy(sp, dev)
    frame = ops.Frame(ops.context(dev))
    cfg = ops.render_cfg(3, mip=True)
    img = torch.empty(cam.height, cam.width, 4, device=dev)
    vis = torch.empty(n, device=dev)
    vc = torch.empty(n, 10, device=dev)
    v_host = (np.random.default_rng(11).standard_normal((cam.height, cam.width, 4)) * 1e-3).astype(np.float32)
    v_out = torch.from_numpy(v_host).to(dev)
    stream = torch.cuda.current_stream(dev)

    def step(hook=None, upstream=v_out, ready=None):
        out = ops.render_stages(cam, cfg, splats.transforms, splats.sh_coeffs, splats.raw_opacities, frame, img, vis,
                                hook=hook)
        if ready is not None:  # the upstream gradient's upload, overlapped with the forward
            stream.wait_event(ready)
        r = ops.rasterize_bwd(out.frame, out.out_img, upstream, vc)
        if hook:
            hook("raster_bwd")
        return r

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    ctx = ops.context(dev)
    l0 = ctx.launch_count
    gpu_uuid = str(torch.cuda.get_device_properties(dev).uuid)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(gpu_uuid if gpu_uuid.startswith("GPU-") else f"GPU-{gpu_uuid}") as clk:
        torch.cuda.synchronize()
        clk.mark("start")
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
        clk.mark("stop")
    ms = e0.elapsed_time(e1)
    launches = (ctx.launch_count - l0) // max(args.steps, 1)
    # per-stage medians
    acc = {}
    for _ in range(5):
        evs = [("start", torch.cuda.Event(enable_timing=True))]
        evs[0][1].record(stream)

        def hook(name):
            e = torch.cuda.Event(enable_timing=True)
            e.record(stream)
            evs.append((name, e))
        step(hook)
        torch.cuda.synchronize()
        for (_, ea), (b, eb) in zip(evs[:-1], evs[1:]):
            acc.setdefault(b, []).append(ea.elapsed_time(eb))
    nv, ni = frame.num_visible, frame.num_intersections
    p, tcount = cam.width * cam.height, cam.num_tiles
    peak, which = peaks()
    stages, roof = {}, {}
    for k, t in acc.items():
        m = statistics.median(t)
        b = stage_bytes(k, n, nv, ni, p, tcount)
        stages[k] = {"ms": round(m, 4), "gbs": round(b / (m / 1e3) / 1e9, 1), "frac": round(b / (m / 1e3) / 1e9 / peak, 4)}
        if k in ("raster_fwd", "raster_bwd"):
            roof[k] = {"bound": "hbm", "kernel": k + "_kernel", "achieved": stages[k]["gbs"], "peak": peak,
                       "unit": "GB/s", "frac": stages[k]["frac"], "traffic": None, "peak_source": which,
                       "alg_bytes": b}
    # end to end: the upstream gradient from pinned host memory each step (on a
    # side stream into one of two device buffers, overlapped with the forward;
    # the backward waits for it), a scalar of the result read back
    pinned = torch.from_numpy(v_host).pin_memory()
    bufs = [torch.empty_like(v_out), torch.empty_like(v_out)]
    done = [None, None]
    copy_stream = torch.cuda.Stream(dev)
    res_host = torch.empty((), dtype=torch.float32).pin_memory()

    def e2e_step(k):
        b = k % 2
        with torch.cuda.stream(copy_stream):
            if done[b] is not None:  # the backward two steps back has read this buffer
                copy_stream.wait_event(done[b])
            bufs[b].copy_(pinned, non_blocking=True)
            ready = copy_stream.record_event()
        r = step(upstream=bufs[b], ready=ready)
        done[b] = stream.record_event()
        res_host.copy_(r.sum(), non_blocking=True)
    for k in range(3):
        e2e_step(k)
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    copy_stream.wait_stream(stream)  # no upload of the timed steps starts before the timed region
    for k in range(args.steps):
        e2e_step(k)
    f1.record(stream)
    torch.cuda.synchronize()
    e2e = {"value": round(args.steps / (f0.elapsed_time(f1) / 1e3), 3), "unit": "steps/s",
           "h2d_bytes_per_step": int(v_out.numel() * 4), "d2h_bytes_per_step": 4,
           "api": "vs_render_project/bin/rasterize + vs_rasterize_backward (ops.render_stages, ops.rasterize_bwd)"}
    out = {"metric": "single-view render fwd+bwd steps/s @1M splats 1920×1080; raster fwd/bwd HBM GB/s vs peak",
           "value": round(args.steps / (ms / 1e3), 3), "unit": "steps/s", "n_gpus": 1, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
           "scaling": "replicas only", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
           "config": {"workload": "configs[1]: 1M SH-3 splats, one 1920x1080 view at distance 6, fx=fy=1600, "
                                  "Mip mode, upstream gradient N(0,1e-3)", "splats": n, "visible": nv,
                      "intersections": ni, "l2": "inputs larger than L2 (params 236 MB, image + gradient 66 MB)"},
           "gpu_launches": int(launches), "clocks": clk.summary(), "stages": stages,
           "roofline": roof["raster_bwd"], "roofline_raster": roof, "e2e": e2e}
    if not args.no_cpu_baseline:
        cores = oracle.set_num_threads(os.cpu_count() or 1)
        t0 = time.perf_counter()
        cfg_o = oracle.make_cfg(3, mip=True)
        ref = oracle.render_forward(cam, cfg_o, sp)
        vc_ref = oracle.raster_bwd(cam, (0.0, 0.0, 0.0), ref["proj"], ref["binning_after"], ref["out_img"], v_host)
        dt = time.perf_counter() - t0
        step()
        torch.cuda.synchronize()
        g_img, g_vc = img.cpu().numpy(), vc[:nv].cpu().numpy()
        out["parity"] = {
            "counts_equal": bool(nv == ref["proj"]["num_visible"] and ni == ref["proj"]["num_isect"]),
            "keys_equal": bool(np.array_equal(frame.field("isect_tile").cpu().numpy().view(np.uint32),
                                              ref["binning"]["tile_ids"]) and
                               np.array_equal(frame.field("isect_compact").cpu().numpy().view(np.uint32),
                                              ref["binning"]["isect_compact"])),
            "ranges_equal": bool(np.array_equal(frame.field("tile_ranges").cpu().numpy().view(np.uint32).reshape(-1, 2),
                                                ref["tile_offsets_pre"]) and
                                 np.array_equal(frame.field("tile_used_end").cpu().numpy().view(np.uint32),
                                                ref["tile_offsets"][:, 1])),
            "img_max_rel": mixed_rel(g_img, ref["out_img"]), "img_px_over_1e-4": count_over(g_img, ref["out_img"]),
            "visible_equal": bool(np.array_equal(vis.cpu().numpy(), ref["visible"])),
            "vcomb_max_rel": mixed_rel(g_vc, vc_ref), "vcomb_over_1e-4": count_over(g_vc, vc_ref)}
        out["cpu_baseline"] = {"value": round(1.0 / dt, 5), "unit": "steps/s", "cores": cores, "kind": "port",
                               "sample": "1 forward + backward of the same view by the C++ oracle (OpenMP)"}
    print(json.dumps(out), flush=True)



def run_sort_stress(args):
    """Benchmark configuration 4 (sort/overlap stress): 10M splats with large
    footprints (log-scales N(-2.5, 0.5), opacity logits N(1, 1), configs[2]
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
           "config": {"workload": "configs[4]: 10M SH-3 splats, log-scales N(-2.5,0.5), opacity logits N(1,1), one "
                                  "3840x2160 view, fx=fy=3000, project+bin+raster fwd+raster bwd (N(0,1e-3) upstream)",
                      "splats": n, "visible": visible, "intersections": isect,
                      "l2": "inputs larger than L2"},
           "stages": {k: {"ms": round(v, 3)} for k, v in ms.items()},
           "roofline": {"bound": "hbm", "kernel": "bin", "achieved": round(bin_bytes / (ms["bin"] / 1e3) / 1e9, 1),
                        "peak": peak, "unit": "GB/s", "frac": round(bin_bytes / (ms["bin"] / 1e3) / 1e9 / peak, 4),
                        "traffic": None, "peak_source": which},
           "clocks": clk.summary()}
    if not args.no_cpu_baseline:
        out["checks"] = sort_stress_checks(frame, cam, cfg, sp)
    print(json.dumps(out), flush=True)


def sort_stress_checks(frame, cam, cfg, sp):
    """Checks of the last render at full size: the projection (visible set,
    per-splat tile counts, depths) against the CPU oracle's bit for bit, and
    size-independent properties of the binning (keys sorted by (tile, depth),
    the tile ranges partition the list, every splat emitted exactly its tile
    count, and the total equals the sum of the counts)."""
    import torch
    import oracle
    oracle.set_num_threads(os.cpu_count() or 1)
    ref = oracle.project(cam, oracle.make_cfg(3, mip=True), sp.transforms, sp.sh, sp.raw_opac)
    nv, ni = frame.num_visible, frame.num_intersections
    res = {"counts_equal": bool(nv == ref["num_visible"] and ni == ref["num_isect"]),
           "compact_from_global_equal": bool(np.array_equal(
               frame.field("compact_from_global").cpu().numpy().view(np.uint32), ref["compact_from_global"])),
           "tile_counts_equal": bool(np.array_equal(frame.field("tile_counts").cpu().numpy().view(np.uint32),
                                                    ref["tile_counts_compact"])),
           "depths_equal": bool(np.array_equal(frame.field("depths").cpu().numpy().view(np.uint32),
                                               ref["depths"].view(np.uint32)))}
    del ref
    tiles = frame.field("isect_tile").long()
    cid = frame.field("isect_compact").long()
    dbits = frame.field("depths").view(torch.int32).long()[cid]
    res["keys_sorted"] = bool(((tiles[1:] > tiles[:-1]) | ((tiles[1:] == tiles[:-1]) & (dbits[1:] >= dbits[:-1])))
                              .all().item())
    del dbits
    T = cam.num_tiles
    hist = torch.bincount(tiles, minlength=T)
    rng = frame.field("tile_ranges").long().view(-1, 2)
    starts = torch.cumsum(hist, 0) - hist
    res["ranges_partition"] = bool(torch.equal(rng[:, 0], starts) and torch.equal(rng[:, 1] - rng[:, 0], hist))
    per = torch.bincount(cid, minlength=nv)
    res["emitted_equals_counts"] = bool(torch.equal(per, frame.field("tile_counts").long()))
    res["total_equals_sum"] = bool(int(frame.field("tile_counts").long().sum().item()) == ni)
    res["what"] = "projection vs the C++ oracle (bit-exact); binning invariants on the GPU at full size"
    return res


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    elif args.config == 1:
        run_microbench(args)
    elif args.config == 4:
        run_sort_stress(args)
    elif args.emulate_peers:
        run_peer_emulation(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
