"""Dataset feed: views, packing and the staged loader.

Mirrors crates/splat-train-dataset: `view_to_packed_data` (src/scene.rs:
113-161), `SceneBatch` (:165-191), `SceneLoader` (src/scene_loader.rs:59-184)
and `LoadDatasetConfig::max_scene_batch_cache_size` (src/config.rs:8-10,
59-61).  Images arrive decoded (8-bit L, LA, RGB or RGBA numpy arrays; the
reference's image decoding is not part of this path).  Packing runs on the
GPU (`vs_pack_view`); `SceneLoader` is the native feed (`vs_feed_*`): pinned
host slots filled by worker threads, a copy stream and the packing kernel,
`ring_slots` batches ahead of the trainer, with packed views kept resident in
HBM up to the cache budget.

Differences from the reference, on purpose: one deterministic visiting order
(epochs of seeded shuffles from the feed's own generator) instead of several
loader tasks each drawing their own order; the cache holds packed views in
device memory rather than host memory.
"""
from __future__ import annotations

import ctypes
import enum
from dataclasses import dataclass

import numpy as np
import torch

from . import _native as N
from . import ops
from .camera import Camera
from .peer import _DeviceArray
from .trainer import SceneBatch

DEFAULT_MAX_SCENE_BATCH_CACHE_SIZE = 6 << 30  # config.rs:8 ("6GiB")
DEFAULT_RING_SLOTS = 4  # scene_loader.rs:69 (channel of 4)


class AlphaMode(enum.IntEnum):
    """crates/splat-train-render/src/lib.rs:121-125."""

    MASKED = 0
    TRANSPARENT = 1


def _as_hwc(image: np.ndarray) -> np.ndarray:
    px = np.ascontiguousarray(image)
    if px.dtype != np.uint8:
        raise TypeError(f"8-bit images only (got {px.dtype})")
    if px.ndim == 2:
        px = px[..., None]
    if px.ndim != 3 or not 1 <= px.shape[2] <= 4:
        raise ValueError(f"image of shape {image.shape}: want [H, W] or [H, W, C] with C in 1..4")
    return px


def view_to_packed_data(image: np.ndarray | torch.Tensor, alpha_mode: AlphaMode, device) -> tuple[torch.Tensor, bool]:
    """Packs a decoded view to `[H, W]` int32 RGBA8 words on the device
    (scene.rs:113-161) and returns (packed, has_alpha)."""
    dev = torch.device(device)
    if isinstance(image, torch.Tensor):
        src = image.to(dev, torch.uint8).contiguous()
        if src.dim() == 2:
            src = src.unsqueeze(-1)
    else:
        src = torch.from_numpy(_as_hwc(image)).to(dev)
    if src.dim() != 3 or not 1 <= src.shape[2] <= 4:
        raise ValueError(f"image of shape {tuple(src.shape)}: want [H, W] or [H, W, C] with C in 1..4")
    h, w, c = src.shape
    out = torch.empty(h, w, dtype=torch.int32, device=dev)
    ctx = ops.context(dev)
    has_alpha = ctypes.c_int32(0)
    ctx.check(ctx.lib.vs_pack_view(ctx.h, ops._ptr(src), w, h, c, int(alpha_mode), ops._ptr(out),
                                   ctypes.byref(has_alpha)))
    return out, bool(has_alpha.value)


@dataclass
class SceneView:
    """One training view: decoded 8-bit pixels and its camera (scene.rs)."""

    image: np.ndarray
    camera: Camera
    alpha_mode: AlphaMode = AlphaMode.MASKED


@dataclass
class Scene:
    views: list


@dataclass
class LoadDatasetConfig:
    max_scene_batch_cache_size: int = DEFAULT_MAX_SCENE_BATCH_CACHE_SIZE


def visiting_order(seed: int, num_views: int, count: int) -> list[int]:
    """The first `count` view indices a loader with this seed visits (host
    only): epochs, each a shuffle of all views."""
    out = np.zeros(max(count, 1), np.uint32)
    st = N.lib().vs_feed_order(ctypes.c_uint64(seed & (2 ** 64 - 1)), num_views, count, out.ctypes.data)
    if st != 0:
        raise ValueError(f"visiting_order({seed}, {num_views}, {count}): status {st}")
    return out[:count].tolist()


class SceneLoader:
    """Hands out `SceneBatch`es with device-resident packed ground truth,
    staged `ring_slots` batches ahead (scene_loader.rs:59-125).

    A batch k that was not served from the HBM cache is valid (in stream order
    on the current torch stream) until the call that hands out batch k + hold:
    `hold` is how many batches a step uses at once.  `views` may be the whole scene or, in a
    view-parallel job, one rank's share (`shard`)."""

    def __init__(self, scene: Scene, seed: int, config: LoadDatasetConfig | None = None, device="cuda",
                 ring_slots: int = DEFAULT_RING_SLOTS, workers: int = 0, hold: int = 1):
        cfg = config or LoadDatasetConfig()
        if not scene.views:
            raise ValueError("SceneLoader needs at least one view")
        self.device = torch.device(device)
        self.ctx = ops.context(self.device)
        self.views = list(scene.views)
        self._pixels = [_as_hwc(v.image) for v in self.views]  # kept alive for the feed's workers
        c = N.FeedCfg()
        c.num_views, c.ring_slots, c.workers, c.hold = len(self.views), int(ring_slots), int(workers), int(hold)
        c.cache_bytes, c.seed = int(cfg.max_scene_batch_cache_size), int(seed) & (2 ** 64 - 1)
        h = ctypes.c_void_p()
        self.ctx.check(self.ctx.lib.vs_feed_create(self.ctx.h, ctypes.byref(c), ctypes.byref(h)))
        self.h = h
        for i, (v, px) in enumerate(zip(self.views, self._pixels)):
            hh, ww, ch = px.shape
            self.ctx.check(self.ctx.lib.vs_feed_set_view(self.h, i, px.ctypes.data, ww, hh, ch, int(v.alpha_mode)))
        self.last_h2d_bytes = 0
        self.last_cached = False
        self.h2d_bytes_total = 0  # host-to-device bytes of all batches handed out

    def next_batch(self) -> SceneBatch:
        b = N.SceneBatchC()
        self.ctx = ops.context(self.device)  # binds the current torch stream: the batch is ready on it
        self.ctx.check(self.ctx.lib.vs_feed_next(self.h, ctypes.byref(b)))
        arr = _DeviceArray(b.img_packed, b.width * b.height, torch.int32)
        img = torch.as_tensor(arr, device=self.device).view(b.height, b.width)
        self.last_h2d_bytes, self.last_cached = int(b.h2d_bytes), bool(b.cached)
        self.h2d_bytes_total += self.last_h2d_bytes
        view = self.views[b.view_index]
        return SceneBatch(img, view.camera, int(b.view_index), has_alpha=bool(b.has_alpha),
                          alpha_mode=AlphaMode(b.alpha_mode))

    def close(self):
        if getattr(self, "h", None):
            self.ctx.lib.vs_feed_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def shard(scene: Scene, rank: int, world: int) -> Scene:
    """Views of one rank in a view-parallel job (round-robin)."""
    return Scene(scene.views[rank::world])
