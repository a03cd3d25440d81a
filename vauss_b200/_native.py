"""ctypes binding of libvauss_b200.so (the C ABI in include/vauss_b200.h).

The library is built in-tree by ``vauss_b200.build``; importing this module
never falls back to anything else: if the library is missing or fails to load,
``lib()`` raises.
"""
from __future__ import annotations

import ctypes
import os

from .camera import VsCamera

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_lib", "libvauss_b200.so")

c_f32p = ctypes.POINTER(ctypes.c_float)
c_u32p = ctypes.POINTER(ctypes.c_uint32)
c_vp = ctypes.c_void_p

STATUS = {0: "VS_OK", 1: "VS_ERR_INVALID", 2: "VS_ERR_CAPACITY", 3: "VS_ERR_CUDA", 4: "VS_ERR_DEVICE_TIMEOUT",
          5: "VS_ERR_UNSUPPORTED"}

FIELDS = dict(compact_from_global=0, global_from_compact=1, depths=2, tile_counts=3, projected=4, depth_order=5,
              isect_tile=6, isect_compact=7, tile_ranges=8, tile_used_end=9, opacities=10, max_radius=11)


class VsError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS.get(status, status)}: {message}")
        self.status = status


class RenderCfg(ctypes.Structure):
    _fields_ = [("mip", ctypes.c_int32), ("sh_degree", ctypes.c_int32), ("sh_half", ctypes.c_int32),
                ("has_min_scale", ctypes.c_int32), ("log_scale_offset", ctypes.c_float),
                ("bg", ctypes.c_float * 3)]


class RenderCounts(ctypes.Structure):
    _fields_ = [("num_visible", ctypes.c_uint32), ("num_tiles", ctypes.c_uint32),
                ("num_intersections", ctypes.c_uint64)]


class AdamCfg(ctypes.Structure):
    _fields_ = [("beta1", ctypes.c_float), ("beta2", ctypes.c_float), ("inv1", ctypes.c_float),
                ("inv2", ctypes.c_float), ("epsilon", ctypes.c_float), ("lr_opac", ctypes.c_float),
                ("opac_reg", ctypes.c_float), ("round_seed", ctypes.c_uint32)]


class Q8Tensor(ctypes.Structure):
    _fields_ = [("m_codes", c_vp), ("v_codes", c_vp), ("m_scales", c_vp), ("v_scales", c_vp)]


PEER_MAX = 8


class IpcHandle(ctypes.Structure):
    _fields_ = [("bytes", ctypes.c_uint8 * 64)]


class PeerSet(ctypes.Structure):
    _fields_ = [("world", ctypes.c_uint32), ("rank", ctypes.c_uint32), ("grads", c_vp * PEER_MAX),
                ("vis", c_vp * PEER_MAX), ("transforms", c_vp * PEER_MAX), ("sh_coeffs", c_vp * PEER_MAX),
                ("raw_opacities", c_vp * PEER_MAX), ("row_format", ctypes.c_uint32), ("views", ctypes.c_uint32),
                ("cams", c_vp * PEER_MAX), ("view_masks", c_vp * PEER_MAX)]


COMPACT_ROW = 16  # VS_COMPACT_ROW: floats per splat of vs_vjp_compact


class RefineCfg(ctypes.Structure):
    _fields_ = [("min_opacity", ctypes.c_float), ("max_bound", ctypes.c_float), ("center", ctypes.c_float * 3),
                ("split_at_screen_size", ctypes.c_float)]


class FeedCfg(ctypes.Structure):
    _fields_ = [("num_views", ctypes.c_uint32), ("ring_slots", ctypes.c_uint32), ("workers", ctypes.c_uint32),
                ("hold", ctypes.c_uint32), ("cache_bytes", ctypes.c_uint64), ("seed", ctypes.c_uint64)]


class SceneBatchC(ctypes.Structure):
    _fields_ = [("img_packed", c_vp), ("width", ctypes.c_uint32), ("height", ctypes.c_uint32),
                ("view_index", ctypes.c_uint32), ("has_alpha", ctypes.c_int32), ("alpha_mode", ctypes.c_int32),
                ("cached", ctypes.c_int32), ("h2d_bytes", ctypes.c_uint64)]


class Q8Cfg(ctypes.Structure):
    _fields_ = [("beta1", ctypes.c_float), ("beta2", ctypes.c_float), ("inv1", ctypes.c_float),
                ("inv2", ctypes.c_float), ("epsilon", ctypes.c_float), ("lr_transforms", ctypes.c_float * 10),
                ("lr_sh_dc", ctypes.c_float), ("lr_sh_rest", ctypes.c_float), ("lr_opac", ctypes.c_float),
                ("opac_reg", ctypes.c_float), ("seed", ctypes.c_uint32), ("noise_scale", ctypes.c_float),
                ("noise_limit", ctypes.c_float), ("noise_seed", ctypes.c_uint32)]


_SIGS = {
    "vs_version": ([], ctypes.c_char_p),
    "vs_ctx_create": ([ctypes.c_int, ctypes.POINTER(c_vp)], ctypes.c_int),
    "vs_ctx_destroy": ([c_vp], None),
    "vs_ctx_set_stream": ([c_vp, c_vp], ctypes.c_int),
    "vs_ctx_last_error": ([c_vp], ctypes.c_char_p),
    "vs_ctx_workspace_bytes": ([c_vp], ctypes.c_uint64),
    "vs_ctx_launch_count": ([c_vp], ctypes.c_uint64),
    "vs_frame_create": ([c_vp, ctypes.POINTER(c_vp)], ctypes.c_int),
    "vs_frame_destroy": ([c_vp], None),
    "vs_frame_buffer": ([c_vp, ctypes.c_int32, ctypes.POINTER(c_vp), ctypes.POINTER(ctypes.c_uint64)], ctypes.c_int),
    "vs_frame_counts": ([c_vp, ctypes.POINTER(RenderCounts)], ctypes.c_int),
    "vs_frame_copy": ([c_vp, ctypes.c_int32, c_vp, ctypes.c_uint64], ctypes.c_int),
    "vs_render_forward": ([c_vp, c_vp, ctypes.POINTER(VsCamera), ctypes.POINTER(RenderCfg), ctypes.c_uint32, c_vp,
                           c_vp, c_vp, c_vp, c_vp, c_vp, ctypes.POINTER(RenderCounts)], ctypes.c_int),
    "vs_render_project": ([c_vp, c_vp, ctypes.POINTER(VsCamera), ctypes.POINTER(RenderCfg), ctypes.c_uint32, c_vp,
                           c_vp, c_vp, c_vp, ctypes.POINTER(RenderCounts)], ctypes.c_int),
    "vs_render_bin": ([c_vp, c_vp], ctypes.c_int),
    "vs_render_rasterize": ([c_vp, c_vp, c_vp, c_vp], ctypes.c_int),
    "vs_render_image": ([c_vp, c_vp, ctypes.POINTER(VsCamera), ctypes.POINTER(RenderCfg), ctypes.c_uint32, c_vp, c_vp,
                         c_vp, c_vp, c_vp, ctypes.POINTER(RenderCounts)], ctypes.c_int),
    "vs_loss": ([c_vp, ctypes.c_uint32, ctypes.c_uint32, c_vp, c_vp, ctypes.c_float, ctypes.c_float, c_vp, c_vp,
                 c_vp], ctypes.c_int),
    "vs_rasterize_backward": ([c_vp, c_vp, c_vp, c_vp, c_vp], ctypes.c_int),
    "vs_project_update": ([c_vp, c_vp, ctypes.POINTER(RenderCfg), ctypes.c_uint32, c_vp, c_vp, c_vp, c_vp, c_vp,
                           c_vp, c_f32p, c_vp, ctypes.POINTER(AdamCfg), c_vp, c_vp, c_vp, c_vp, ctypes.c_int32],
                          ctypes.c_int),
    "vs_sh_step": ([c_vp, ctypes.c_uint32, ctypes.c_uint32, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_f32p,
                    ctypes.c_float, ctypes.c_float, ctypes.c_float, ctypes.c_float, ctypes.c_float, ctypes.c_float,
                    ctypes.c_uint32], ctypes.c_int),
    "vs_step_q8": ([c_vp, c_vp, ctypes.POINTER(RenderCfg), ctypes.c_uint32, c_vp, c_vp, c_vp, c_vp, c_vp, Q8Tensor,
                    Q8Tensor, Q8Tensor, ctypes.POINTER(Q8Cfg), c_vp, c_vp, c_vp, c_vp], ctypes.c_int),
    "vs_vjp_dense": ([c_vp, c_vp, ctypes.POINTER(RenderCfg), ctypes.c_uint32, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp,
                      c_vp, c_vp, c_vp], ctypes.c_int),
    "vs_vjp_compact": ([c_vp, c_vp, ctypes.POINTER(RenderCfg), ctypes.c_uint32, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp,
                        c_vp, c_vp, c_vp, c_vp, ctypes.c_uint32, c_vp], ctypes.c_int),
    "vs_adam_q8_dense": ([c_vp, ctypes.c_uint32, ctypes.c_int32, c_vp, c_vp, c_vp, c_vp, Q8Tensor, Q8Tensor,
                          Q8Tensor, ctypes.POINTER(Q8Cfg), c_vp, c_vp], ctypes.c_int),
    "vs_peer_alloc": ([c_vp, ctypes.c_uint64, ctypes.POINTER(c_vp), ctypes.POINTER(IpcHandle)], ctypes.c_int),
    "vs_peer_free": ([c_vp, c_vp], ctypes.c_int),
    "vs_peer_open": ([c_vp, ctypes.POINTER(IpcHandle), ctypes.POINTER(c_vp)], ctypes.c_int),
    "vs_peer_close": ([c_vp, c_vp], ctypes.c_int),
    "vs_peer_barrier": ([c_vp, ctypes.POINTER(c_vp), ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32],
                        ctypes.c_int),
    "vs_ctx_check": ([c_vp], ctypes.c_int),
    "vs_adam_q8_peer": ([c_vp, ctypes.c_uint32, ctypes.c_int32, ctypes.c_uint32, ctypes.c_uint32,
                         ctypes.POINTER(PeerSet), Q8Tensor, Q8Tensor, Q8Tensor, ctypes.POINTER(Q8Cfg)], ctypes.c_int),
    "vs_refine_table": ([c_vp, ctypes.c_uint32, c_vp, c_vp, ctypes.c_uint32, ctypes.c_int32, c_vp, c_vp, c_vp, c_vp,
                         ctypes.POINTER(RefineCfg), c_vp], ctypes.c_int),
    "vs_refine_split": ([c_vp, ctypes.c_uint32, c_vp, c_vp, ctypes.c_uint32, ctypes.c_int32, c_vp, ctypes.c_uint32,
                         c_vp, c_vp, c_vp, ctypes.c_float, ctypes.c_float, ctypes.c_uint32, c_vp], ctypes.c_int),
    "vs_q8_reset_rows": ([c_vp, Q8Tensor, ctypes.c_uint32, ctypes.c_uint32, c_vp], ctypes.c_int),
    "vs_opacity_decay": ([c_vp, ctypes.c_uint32, c_vp, ctypes.c_float], ctypes.c_int),
    "vs_min_scale": ([c_vp, ctypes.c_uint32, c_vp, c_vp, ctypes.c_uint32, ctypes.c_float, c_vp], ctypes.c_int),
    "vs_fold_min_scale": ([c_vp, ctypes.c_uint32, c_vp, c_vp, c_vp], ctypes.c_int),
    "vs_pack_view": ([c_vp, c_vp, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_int32, c_vp,
                      ctypes.POINTER(ctypes.c_int32)], ctypes.c_int),
    "vs_feed_create": ([c_vp, ctypes.POINTER(FeedCfg), ctypes.POINTER(c_vp)], ctypes.c_int),
    "vs_feed_set_view": ([c_vp, ctypes.c_uint32, c_vp, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32,
                          ctypes.c_int32], ctypes.c_int),
    "vs_feed_next": ([c_vp, ctypes.POINTER(SceneBatchC)], ctypes.c_int),
    "vs_feed_destroy": ([c_vp], None),
    "vs_feed_order": ([ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint32, c_vp], ctypes.c_int),
    "vs_ply_row_bytes": ([ctypes.c_int32], ctypes.c_uint64),
    "vs_ply_encode": ([c_vp, ctypes.c_uint32, ctypes.c_int32, c_vp, c_vp, ctypes.c_int32, c_vp, c_vp], ctypes.c_int),
    "vs_ply_decode": ([c_vp, ctypes.c_uint32, c_vp, ctypes.c_uint32, ctypes.c_uint32, c_vp, c_vp, c_vp, c_vp, c_vp],
                      ctypes.c_int),
    "vs_gather_stats": ([c_vp, ctypes.c_uint32, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp], ctypes.c_int),
    "vs_noise_means": ([c_vp, ctypes.c_uint32, c_vp, c_vp, c_vp, ctypes.c_float, ctypes.c_float, ctypes.c_uint32],
                       ctypes.c_int),
    "vs_radix_sort_pairs": ([c_vp, c_vp, c_vp, ctypes.c_uint32, ctypes.c_uint32], ctypes.c_int),
    "vs_radix_sort_pairs_static": ([c_vp, c_vp, c_vp, ctypes.c_uint32, ctypes.c_uint32], ctypes.c_int),
    "vs_scan_inclusive": ([c_vp, c_vp, ctypes.c_uint32, c_vp], ctypes.c_int),
    "vs_math_probe": ([c_vp, ctypes.c_int32, c_vp, c_vp, ctypes.c_uint32], ctypes.c_int),
}

EXPORTED = tuple(_SIGS.keys())

_lib = None


def lib() -> ctypes.CDLL:
    """Load libvauss_b200.so; raises if it is missing (no fallback exists)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m vauss_b200.build`")
        L = ctypes.CDLL(LIB_PATH)
        for name, (args, res) in _SIGS.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def check(ctx, status: int):
    if status != 0:
        msg = lib().vs_ctx_last_error(ctx).decode() if ctx else ""
        raise VsError(status, msg)
