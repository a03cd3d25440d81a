"""One rank of the two-GPU check in test_gpu_multi.py (run under torchrun).

Runs a few view-parallel steps twice from the same splats: through peer
memory (sharded fused Adam over NVLink) and through one NCCL all-reduce of the
dense rows followed by the replicated Adam.  The exchanges themselves agree
bit for bit (two rows add as a + b either way), but the rasterizer backward
sums per-splat gradients with float atomics, so two renders of one view can
round differently: the two paths are compared with the tolerance of the
single-GPU training test.  The replicas of the two ranks must be identical.
"""
import os
import sys
from datetime import timedelta

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from vauss_b200 import ops, scenes  # noqa: E402
from vauss_b200.peer import PeerGroup, gather_bytes_nccl  # noqa: E402
from vauss_b200.trainer import SceneBatch, Splats, TrainConfig  # noqa: E402
from vauss_b200.view_parallel import ViewParallelTrainer  # noqa: E402


def main():
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    dev = torch.device(f"cuda:{local}")
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    sp, cams = scenes.config_train(seed=5, n=60_000, views=8)
    tgt = scenes.random_splats(60_000, 99, mean_lo=-5.0, mean_hi=5.0, log_scale_mu=-4.5, log_scale_sigma=0.6,
                               opac_mu=0.0, opac_sigma=1.5, sh_degree=3)
    ts = Splats.from_numpy(tgt, dev)
    gts = []
    for cam in cams:
        out = ops.render(cam, ops.render_cfg(3, mip=True), ts.transforms, ts.sh_coeffs, ts.raw_opacities)
        gts.append(torch.from_numpy(scenes.pack_rgba8(out.out_img[..., :3].clamp(0, 1).cpu().numpy()).view(np.int32)).to(dev))
    cfg = TrainConfig(optimizer="q8")
    kw = dict(scene_extent=8.0, median_scale=0.02, seed=3)
    peer = PeerGroup(dev, world, rank, lambda b: gather_bytes_nccl(b, dev))
    a = ViewParallelTrainer(cfg, dev, peer=peer, **kw)
    b = ViewParallelTrainer(cfg, dev, **kw)
    sa = a.adopt(Splats.from_numpy(sp, dev))
    sb = Splats.from_numpy(sp, dev)
    bad = []
    for step in range(4):
        v = (step * world + rank) % len(cams)
        batch = [SceneBatch(gts[v], cams[v], v)]
        sa, la = a.step_views(batch, sa)
        sb, lb = b.step_views(batch, sb)
        torch.cuda.synchronize(dev)
        for name, x, y in (("transforms", sa.transforms, sb.transforms), ("sh", sa.sh_coeffs, sb.sh_coeffs),
                           ("opacity", sa.raw_opacities, sb.raw_opacities)):
            err = (x - y).abs()
            bound = 2e-5 + 1e-4 * y.abs()
            frac = float((err > bound).float().mean())
            worst = float(err.max())
            if frac > 1e-4 or worst > 2e-4 + 1e-3 * float(y.abs().max()):
                bad.append(f"rank {rank} step {step} {name}: {frac:.2e} of values out of tolerance, max {worst:.3g}")
        if abs(float(la.loss) - float(lb.loss)) > 1e-5 * max(1.0, abs(float(lb.loss))):
            bad.append(f"rank {rank} step {step} loss {float(la.loss)} vs {float(lb.loss)}")
    # the replicas of the two ranks are identical (every shard owner wrote both)
    mine = torch.cat([sa.transforms.reshape(-1), sa.sh_coeffs.reshape(-1), sa.raw_opacities.reshape(-1)])
    alls = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(alls, mine.clone())
    for r in range(1, world):
        if not torch.equal(alls[0].view(torch.int32), alls[r].view(torch.int32)):
            bad.append(f"replica of rank {r} differs from rank 0's in {int((alls[0] != alls[r]).sum())} values")
    torch.cuda.synchronize(dev)
    dist.barrier()
    peer.check()
    peer.close()
    torch.cuda.synchronize(dev)
    dist.barrier()
    dist.destroy_process_group()
    if bad:
        print("\n".join(bad), flush=True)
        sys.exit(1)
    if rank == 0:
        print("MULTI_GPU_OK", flush=True)


if __name__ == "__main__":
    main()
