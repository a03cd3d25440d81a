"""Checkpoint I/O: PLY export/import of splats, 8-bit moment dumps, and a
resumable trainer checkpoint.

PLY export mirrors `splat_to_ply` (crates/splat-train-serde/src/export.rs:
284-425): binary little-endian, header comments for the vertical axis, the
render mode and the SH degree, one vertex element of f32 properties in the
inria order.  The rows are encoded on the GPU (`vs_ply_encode`).  Import
mirrors `load_splat_from_ply` / `parse_ply` (import.rs:218-229, 269-510): the
header is parsed here, the vertex rows are decoded on the GPU
(`vs_ply_decode`) with the reference's defaults for absent properties
(rotation (1,0,0,0), log-scale -4, raw opacity logit(0.5) = 0, SH 0.5 for a
file without colour), `red/green/blue` (or r/g/b) overriding the DC
coefficients, and every k-th row kept with `subsample_points` k.
The SuperSplat compressed layout (a `chunk` element first) and non-little-
endian files are rejected with an error.

The reference does not persist optimizer moments; here `save_moments` /
`load_moments` dump the 8-bit m and v codes and their block scales verbatim,
and `save_checkpoint` / `load_checkpoint` add the trainer state needed to
continue a run (step count, Adam time, RNG state, refine statistics and the
refiner's state).
"""
from __future__ import annotations

import dataclasses
import json
import os
import struct
from dataclasses import dataclass

import numpy as np
import torch

from . import _native as N
from . import ops

SH_C0 = 0.28209479177387814  # crates/splat-train-render/src/sh.rs
_TYPES = {"char": "i1", "int8": "i1", "uchar": "u1", "uint8": "u1", "short": "i2", "int16": "i2", "ushort": "u2",
          "uint16": "u2", "int": "i4", "int32": "i4", "uint": "u4", "uint32": "u4", "float": "f4", "float32": "f4",
          "double": "f8", "float64": "f8"}
_COLOR = ("red", "green", "blue")
_COLOR_ALIAS = {"r": "red", "g": "green", "b": "blue"}


def _f32_text(v: float) -> str:
    """An f32 the way Rust's Display prints it (shortest round trip, no
    trailing ".0")."""
    return np.format_float_positional(np.float32(v), trim="-")


def ply_property_names(sh_degree: int) -> list[str]:
    rest = (sh_degree + 1) ** 2 - 1
    return (["x", "y", "z", "scale_0", "scale_1", "scale_2", "opacity", "rot_0", "rot_1", "rot_2", "rot_3",
             "f_dc_0", "f_dc_1", "f_dc_2"] + [f"f_rest_{k}" for k in range(3 * rest)])


def ply_header(num_splats: int, sh_degree: int, up_axis=None, render_mode: str = "default") -> bytes:
    """Header of an exported splat PLY (export.rs:291-317)."""
    lines = ["ply", "format binary_little_endian 1.0", "comment Exported from vauss_b200"]
    if up_axis is None:
        lines.append("comment Vertical axis: y")
    else:
        lines.append("comment Vertical axis: " + " ".join(_f32_text(v) for v in up_axis))
    lines += [f"comment SplatRenderMode: {render_mode}", f"comment SH degree: {sh_degree}",
              f"element vertex {num_splats}"]
    lines += [f"property float {p}" for p in ply_property_names(sh_degree)]
    lines.append("end_header")
    return ("\n".join(lines) + "\n").encode("ascii")


def ply_rows(splats, device=None) -> np.ndarray:
    """The vertex rows of `splats` as host f32 [N, 14 + 3 rest], encoded on
    the GPU.  A Mip 3D-filter floor is folded into copies of the scales and
    opacities first, as the reference's export bakes it
    (gaussian_splats.rs:390-402)."""
    t, sh, o = splats.transforms, splats.sh_coeffs, splats.raw_opacities
    if getattr(splats, "min_scale", None) is not None:
        t, o = t.clone(), o.clone()
        ops.fold_min_scale(t, o, splats.min_scale)
    dev = t.device if device is None else torch.device(device)
    n, coeffs = t.shape[0], sh.shape[1]
    degree = int(round(coeffs ** 0.5)) - 1
    row = int(N.lib().vs_ply_row_bytes(degree))
    if row == 0:
        raise ValueError(f"SH degree {degree} cannot be written")
    out = np.empty((n, row // 4), np.float32)
    if n:
        ctx = ops.context(dev)
        ctx.check(ctx.lib.vs_ply_encode(ctx.h, n, degree, ops._ptr(t), ops._ptr(sh), int(sh.dtype == torch.float16),
                                        ops._ptr(o), out.ctypes.data))
    return out


def splat_to_ply(splats, up_axis=None, render_mode: str = "default") -> bytes:
    """The PLY file of `splats` (export.rs:284-318)."""
    header = ply_header(splats.num_splats, splats.sh_degree, up_axis, render_mode)
    return header + ply_rows(splats).tobytes()


def write_ply(path: str, splats, up_axis=None, render_mode: str = "default") -> int:
    """Writes `splats` to `path`; returns the bytes written."""
    header = ply_header(splats.num_splats, splats.sh_degree, up_axis, render_mode)
    rows = ply_rows(splats)
    with open(path, "wb") as f:
        f.write(header)
        f.write(memoryview(rows).cast("B"))
    return len(header) + rows.nbytes


# ---- import ----
@dataclass
class PlyElement:
    name: str
    count: int
    properties: list  # (name, numpy type code)


@dataclass
class ParseMetadata:
    """import.rs:20-25."""

    up_axis: tuple | None
    render_mode: str | None
    total_splats: int
    comments: list


def _parse_header(data: bytes) -> tuple[list, list, int, str]:
    end = data.find(b"end_header")
    if not data.startswith(b"ply") or end < 0:
        raise ValueError("not a PLY file (no 'ply' magic or no end_header)")
    nl = data.find(b"\n", end)
    if nl < 0:
        raise ValueError("truncated PLY header")
    text = data[:end].decode("ascii", errors="replace")
    elements, comments, fmt = [], [], None
    for line in text.splitlines():
        parts = line.strip().split()
        if not parts:
            continue
        if parts[0] == "format":
            fmt = parts[1]
        elif parts[0] == "comment":
            comments.append(line.strip()[len("comment"):].strip())
        elif parts[0] == "element":
            elements.append(PlyElement(parts[1], int(parts[2]), []))
        elif parts[0] == "property":
            if not elements:
                raise ValueError("PLY property before any element")
            if parts[1] == "list":
                elements[-1].properties.append((parts[-1], None))
            else:
                if parts[1] not in _TYPES:
                    raise ValueError(f"PLY property type {parts[1]}")
                elements[-1].properties.append((parts[2], _TYPES[parts[1]]))
    return elements, comments, nl + 1, fmt


def _metadata(comments: list, total: int) -> ParseMetadata:
    """Vertical axis and render mode from the comments, the last one winning
    (import.rs:282-324)."""
    up, mode = None, None
    for c in comments:
        s = c.lower()
        if s.startswith("vertical axis: "):
            suffix = s[len("vertical axis: "):].strip()
            axis = {"x": (1.0, 0.0, 0.0), "y": (0.0, -1.0, 0.0), "z": (0.0, 0.0, -1.0)}.get(suffix)
            if axis is None:
                vals = []
                for p in suffix.replace(",", " ").replace("[", " ").replace("]", " ").split():
                    try:
                        vals.append(float(p))
                    except ValueError:
                        pass
                axis = tuple(vals) if len(vals) == 3 else None
            if axis is not None:
                up = axis
        if s.startswith("splatrendermode: "):
            m = s[len("splatrendermode: "):].strip()
            if m in ("mip", "surfel", "default"):
                mode = m
    return ParseMetadata(up, mode, total, comments)


def _dequant(col: np.ndarray) -> np.ndarray:
    """PlyGaussian's de_quant (ply_gaussian.rs:43-66): u8 / 254, u16 / 65534."""
    if col.dtype == np.uint8:
        return col.astype(np.float32) / np.float32(254.0)
    if col.dtype == np.uint16:
        return col.astype(np.float32) / np.float32(65534.0)
    return col.astype(np.float32)


def load_ply(src, device, subsample_points: int | None = None):
    """Reads a splat PLY (path, bytes or a binary file object) into device
    `Splats`; returns (splats, ParseMetadata)."""
    from .trainer import Splats
    if isinstance(src, (bytes, bytearray, memoryview)):
        data = bytes(src)
    elif isinstance(src, (str, os.PathLike)):
        with open(src, "rb") as f:
            data = f.read()
    else:
        data = src.read()
    elements, comments, body, fmt = _parse_header(data)
    if fmt != "binary_little_endian":
        raise NotImplementedError(f"PLY format {fmt}: only binary_little_endian is read")
    names = [e.name for e in elements]
    if "vertex" not in names:
        raise ValueError("Unknown format: no vertex element")
    if elements[0].name == "chunk":
        raise NotImplementedError("compressed (SuperSplat chunk) PLY files are not read")
    offset = body
    for e in elements[:names.index("vertex")]:
        if any(t is None for _, t in e.properties):
            raise NotImplementedError(f"element {e.name} with list properties before the vertices")
        offset += e.count * int(np.dtype([(n, "<" + t) for n, t in e.properties]).itemsize)
    vert = elements[names.index("vertex")]
    if any(t is None for _, t in vert.properties):
        raise NotImplementedError("list properties in the vertex element")
    dt = np.dtype([(n, "<" + t) for n, t in vert.properties])
    if len(data) < offset + vert.count * dt.itemsize:
        raise ValueError("truncated PLY body")
    rows = np.frombuffer(data, dtype=dt, count=vert.count, offset=offset)
    total = vert.count
    k = int(subsample_points or 1)
    if k > 1:
        rows = rows[k - 1::k][:total // k]
    n = int(rows.shape[0])
    props = {p: t for p, t in vert.properties}
    for a in ("x", "y", "z"):
        if a not in props:
            raise ValueError(f"PLY vertex without '{a}'")
    colors = {}
    for p in props:
        c = _COLOR_ALIAS.get(p, p)
        if c in _COLOR:
            colors[c] = p
    sh_count = sum(1 for p in props if p.startswith("f_rest_") or p.startswith("f_dc_")
                   or p in ("r", "g", "b", "red", "green", "blue"))
    coeffs = sh_count // 3 if sh_count else 1
    if coeffs * 3 != (sh_count or 3) or coeffs not in (1, 4, 9, 16):
        raise ValueError(f"{sh_count} SH properties: not 3 (d+1)^2 for a degree d in 0..3")
    rest = coeffs - 1
    # output value j -> property name (None = default), defaults as the reference
    want = ["x", "y", "z", "rot_0", "rot_1", "rot_2", "rot_3", "scale_0", "scale_1", "scale_2", "opacity"]
    defaults = [0.0, 0.0, 0.0, 1.0, 0.0, 0.0, 0.0, -4.0, -4.0, -4.0, 0.0]
    for kk in range(coeffs):
        for ch in range(3):
            want.append(f"f_dc_{ch}" if kk == 0 else f"f_rest_{ch * rest + kk - 1}")
            defaults.append(0.5 if sh_count == 0 else 0.0)
    use_rgb = len(colors) == 3
    raw_ok = (not use_rgb and dt.itemsize % 4 == 0
              and all(props[w] == "f4" and dt.fields[w][1] % 4 == 0 for w in want if w in props))
    if raw_ok:
        src_rows, row_bytes = np.ascontiguousarray(rows), dt.itemsize
        offsets = [dt.fields[w][1] if w in props else -1 for w in want]
    else:  # non-f32 or unaligned properties, or colours: gather an f32 matrix on the host
        cols = [w for w in want if w in props]
        mat = np.zeros((n, max(len(cols), 1)), np.float32)
        for c, w in enumerate(cols):
            mat[:, c] = rows[w].astype(np.float32)
        offsets = [4 * cols.index(w) if w in props else -1 for w in want]
        if use_rgb:
            dc_pos = [want.index(f"f_dc_{ch}") for ch in range(3)]
            extra = np.zeros((n, 3), np.float32)
            for ch, name in enumerate(_COLOR):
                extra[:, ch] = (_dequant(rows[colors[name]]) - np.float32(0.5)) / np.float32(SH_C0)
            mat = np.concatenate([mat, extra], axis=1)
            for ch in range(3):
                offsets[dc_pos[ch]] = 4 * (mat.shape[1] - 3 + ch)
        src_rows, row_bytes = np.ascontiguousarray(mat), mat.shape[1] * 4
    dev = torch.device(device)
    t = torch.empty(n, 10, device=dev)
    sh = torch.empty(n, coeffs, 3, device=dev)
    o = torch.empty(n, device=dev)
    if n:
        ctx = ops.context(dev)
        off = np.asarray(offsets, np.int32)
        dft = np.asarray(defaults, np.float32)
        ctx.check(ctx.lib.vs_ply_decode(ctx.h, n, src_rows.ctypes.data, row_bytes, coeffs, off.ctypes.data,
                                        dft.ctypes.data, ops._ptr(t), ops._ptr(sh), ops._ptr(o)))
    return Splats(t, sh, o), _metadata(comments, n)


# ---- 8-bit moments ----
_MOM_MAGIC = b"VSQ8MOMS"
_MOM_KEYS = ("t", "sh", "o")


def _pad16(f):
    pad = (-f.tell()) % 16
    if pad:
        f.write(b"\0" * pad)


def save_moments(path_or_file, optim: dict) -> None:
    """Dumps the Q8 moments (t, sh, o: m/v codes and block scales) and the
    Adam time.  Layout: magic, u32 version 1, u32 tensors, u64 time; per
    tensor an 8-byte name, u64 values, u64 blocks; then per tensor m codes,
    v codes, m scales, v scales, each starting on a 16-byte boundary."""
    f = open(path_or_file, "wb") if isinstance(path_or_file, (str, os.PathLike)) else path_or_file
    try:
        f.write(_MOM_MAGIC + struct.pack("<IIQ", 1, len(_MOM_KEYS), int(optim.get("time", 0))))
        for k in _MOM_KEYS:
            m = optim[k]
            f.write(k.encode().ljust(8, b"\0") + struct.pack("<QQ", m.m_codes.numel(), m.m_scales.numel()))
        for k in _MOM_KEYS:
            m = optim[k]
            for arr in (m.m_codes, m.v_codes, m.m_scales, m.v_scales):
                _pad16(f)
                f.write(arr.detach().cpu().numpy().tobytes())
    finally:
        if f is not path_or_file:
            f.close()


def load_moments(path_or_file, device) -> dict:
    f = open(path_or_file, "rb") if isinstance(path_or_file, (str, os.PathLike)) else path_or_file
    try:
        data = f.read()
    finally:
        if f is not path_or_file:
            f.close()
    if not data.startswith(_MOM_MAGIC):
        raise ValueError("not a moment dump")
    version, count, time = struct.unpack_from("<IIQ", data, 8)
    if version != 1 or count != len(_MOM_KEYS):
        raise ValueError(f"moment dump version {version} with {count} tensors")
    pos = 24
    sizes = []
    for _ in range(count):
        name = data[pos:pos + 8].rstrip(b"\0").decode()
        values, blocks = struct.unpack_from("<QQ", data, pos + 8)
        sizes.append((name, values, blocks))
        pos += 24
    dev = torch.device(device)
    out = {"time": int(time)}
    for name, values, blocks in sizes:
        m = ops.Q8Moments.__new__(ops.Q8Moments)
        arrays = []
        for nbytes, dtype in ((values, np.uint8), (values, np.uint8), (4 * blocks, np.float32), (4 * blocks, np.float32)):
            pos += (-pos) % 16
            if pos + nbytes > len(data):
                raise ValueError("truncated moment dump")
            arrays.append(torch.from_numpy(np.frombuffer(data, dtype=dtype, count=nbytes // np.dtype(dtype).itemsize,
                                                         offset=pos).copy()).to(dev))
            pos += nbytes
        m.m_codes, m.v_codes, m.m_scales, m.v_scales = arrays
        out[name] = m
    return out


# ---- trainer checkpoint ----
def save_checkpoint(directory: str, trainer, splats, up_axis=None) -> None:
    """splats.ply + moments.q8 + record.npz + state.json under `directory`."""
    os.makedirs(directory, exist_ok=True)
    write_ply(os.path.join(directory, "splats.ply"), splats, up_axis,
              "mip" if trainer.config.render_mode_mip else "default")
    state = {"config": dataclasses.asdict(trainer.config), "step_count": trainer.step_count,
             "scene_extent": trainer.scene_extent, "median_scale": trainer.median_scale,
             "rng": trainer.rng.bit_generator.state, "train_pixels": trainer.train_pixels,
             "view_centers": None if trainer.view_centers is None else np.asarray(trainer.view_centers).tolist(),
             "view_cams": None if trainer.view_cams is None else trainer.view_cams.cpu().numpy().tolist(),
             "optimizer": trainer.config.optimizer, "refiner": None}
    if trainer.optim is not None:
        if trainer.config.optimizer != "q8":
            raise NotImplementedError("checkpoints hold 8-bit moments; the reference-mode optimizer is not saved")
        save_moments(os.path.join(directory, "moments.q8"), trainer.optim)
    # the PLY holds unit quaternions (as exported); training continues from
    # the raw ones, whose norm enters the rotation gradient
    rec = trainer.record
    extra = {} if rec is None else dict(refine_norm=rec.refine_norm.cpu().numpy(), vis_count=rec.vis_count.cpu().numpy(),
                                        max_screen=rec.max_screen.cpu().numpy())
    if splats.min_scale is not None:  # the PLY holds the folded splat; keep the raw values and the floor
        extra.update(raw_log_scales=splats.transforms[:, 7:10].cpu().numpy(),
                     raw_opacities=splats.raw_opacities.cpu().numpy(), min_scale=splats.min_scale.cpu().numpy())
    np.savez(os.path.join(directory, "record.npz"), raw_rotations=splats.transforms[:, 3:7].cpu().numpy(), **extra)
    r = trainer.refiner
    if r is not None:
        state["refiner"] = {"center": r.bounds.center.tolist(), "extent": r.bounds.extent.tolist(),
                            "far_share": r.far_share, "growth_start_count": r.growth_start_count}
    with open(os.path.join(directory, "state.json"), "w") as f:
        json.dump(state, f)


def load_checkpoint(directory: str, device):
    """Returns (trainer, splats) that continue the saved run."""
    from .refine import Bounds, Refiner
    from .trainer import RefineRecord, SplatTrainer, TrainConfig
    with open(os.path.join(directory, "state.json")) as f:
        state = json.load(f)
    cfg = TrainConfig(**{k: (tuple(v) if isinstance(v, list) else v) for k, v in state["config"].items()})
    dev = torch.device(device)
    tr = SplatTrainer(cfg, dev, scene_extent=state["scene_extent"], median_scale=state["median_scale"])
    tr.step_count = int(state["step_count"])
    tr.rng.bit_generator.state = state["rng"]
    tr.train_pixels = state["train_pixels"]
    tr.view_centers = None if state["view_centers"] is None else np.asarray(state["view_centers"], np.float32)
    splats, _ = load_ply(os.path.join(directory, "splats.ply"), dev)
    rec = np.load(os.path.join(directory, "record.npz"))
    splats.transforms[:, 3:7] = torch.from_numpy(rec["raw_rotations"]).to(dev)
    if "min_scale" in rec.files:
        splats.transforms[:, 7:10] = torch.from_numpy(rec["raw_log_scales"]).to(dev)
        splats.raw_opacities.copy_(torch.from_numpy(rec["raw_opacities"]).to(dev))
        splats.min_scale = torch.from_numpy(rec["min_scale"]).to(dev)
    if state.get("view_cams") is not None:
        tr.view_cams = torch.tensor(state["view_cams"], dtype=torch.float32, device=dev)
    mom = os.path.join(directory, "moments.q8")
    if os.path.exists(mom):
        tr.optim = load_moments(mom, dev)
        tr.record = RefineRecord(*(torch.from_numpy(rec[k]).to(dev) for k in ("refine_norm", "vis_count",
                                                                              "max_screen")))
    if state["refiner"] is not None:
        r = state["refiner"]
        tr.refiner = Refiner(cfg, Bounds(np.asarray(r["center"], np.float32), np.asarray(r["extent"], np.float32)),
                             tr.rng, tr.train_pixels, tr.view_centers)
        tr.refiner.far_share = r["far_share"]
        tr.refiner.growth_start_count = r["growth_start_count"]
    return tr, splats
