"""Pinhole camera and the projection uniforms the kernels take.

Mirrors the reference's ``Camera`` (crates/splat-train-render/src/camera.rs:12-97):
a camera-to-world pose, a focal length and a principal point.  Camera space is
x right, y down, z forward (a splat is in front when its view-space z >= 0.01,
kernels/project_forward.rs:79-82).  ``viewmat`` is the world-to-camera 3x4
matrix in column-major order, the layout of the reference's
``ProjectUniforms`` (kernels/types.rs:53-82): rotation columns, then the
translation column.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np


class VsCamera(ctypes.Structure):
    """C layout of ``vs_camera`` (include/vauss_b200.h)."""

    _fields_ = [
        ("viewmat", ctypes.c_float * 12),
        ("fx", ctypes.c_float),
        ("fy", ctypes.c_float),
        ("cx", ctypes.c_float),
        ("cy", ctypes.c_float),
        ("cam_pos", ctypes.c_float * 3),
        ("img_w", ctypes.c_uint32),
        ("img_h", ctypes.c_uint32),
    ]


@dataclass
class Camera:
    """A pinhole view: world-to-camera rotation ``R`` (3x3), translation ``t``,
    focal lengths and principal point in pixels, and the image size."""

    R: np.ndarray
    t: np.ndarray
    fx: float
    fy: float
    cx: float
    cy: float
    width: int
    height: int

    @property
    def position(self) -> np.ndarray:
        """Camera centre in world space (the view-direction origin of the SH
        colour, kernels/project_visible.rs:36)."""
        return (-self.R.T @ self.t).astype(np.float32)

    @property
    def viewmat(self) -> np.ndarray:
        """World-to-camera 3x4, column-major, 12 floats."""
        m = np.zeros((3, 4), dtype=np.float32)
        m[:, :3] = self.R
        m[:, 3] = self.t
        return np.ascontiguousarray(m.T.reshape(-1))

    @property
    def tile_bounds(self) -> tuple[int, int]:
        return (self.width + 15) // 16, (self.height + 15) // 16

    @property
    def num_tiles(self) -> int:
        tw, th = self.tile_bounds
        return tw * th

    def to_c(self) -> VsCamera:
        c = VsCamera()
        vm = self.viewmat
        for i in range(12):
            c.viewmat[i] = float(vm[i])
        c.fx, c.fy, c.cx, c.cy = float(self.fx), float(self.fy), float(self.cx), float(self.cy)
        p = self.position
        for i in range(3):
            c.cam_pos[i] = float(p[i])
        c.img_w, c.img_h = int(self.width), int(self.height)
        return c


def look_at(position, target, width: int, height: int, fx: float, fy: float | None = None,
            up=(0.0, 0.0, 1.0)) -> Camera:
    """Camera at ``position`` looking at ``target`` with the principal point at
    the image centre (``center_uv = (0.5, 0.5)``, camera.rs:62-67)."""
    p = np.asarray(position, dtype=np.float64)
    f = np.asarray(target, dtype=np.float64) - p
    f /= np.linalg.norm(f)
    upv = np.asarray(up, dtype=np.float64)
    if abs(float(np.dot(f, upv))) > 0.999:
        upv = np.array([0.0, 1.0, 0.0]) if abs(f[1]) < 0.9 else np.array([1.0, 0.0, 0.0])
    right = np.cross(f, upv)
    right /= np.linalg.norm(right)
    down = np.cross(f, right)
    c2w = np.stack([right, down, f], axis=1)  # columns: camera axes in world space
    R = c2w.T
    t = -R @ p
    fy = fx if fy is None else fy
    return Camera(R=R.astype(np.float32), t=t.astype(np.float32), fx=float(fx), fy=float(fy),
                  cx=0.5 * width, cy=0.5 * height, width=int(width), height=int(height))
