"""Checkpoint I/O on the host: the PLY header (the field counts the
reference's export tests check, export.rs:513-541), comment metadata
(import.rs:282-324), the moment dump round trip, and the oracle's row
encoding on the reference tests' splats (test_utils in
crates/splat-train-serde/src/lib.rs:27-72)."""
import io

import numpy as np
import pytest
import torch

import oracle
from vauss_b200 import checkpoint, ops


def reference_test_splats(degree: int, n: int):
    """The values of create_test_splats_with_count: means (i, i+1, i+2),
    identity rotations, log scales -0.1/0.2/-0.3 + 0.05 i, SH per channel
    DC 0.5 + 0.1 i and rest j 0.1 + 0.01 i, raw opacity 0.8 - 0.1 i."""
    coeffs = (degree + 1) ** 2
    t = np.zeros((n, 10), np.float32)
    sh_cm = np.zeros((n, 3, coeffs), np.float32)  # as written there: channel-major per splat
    o = np.zeros(n, np.float32)
    for i in range(n):
        f = np.float32(i)
        t[i, :3] = [f, f + 1, f + 2]
        t[i, 3:7] = [1, 0, 0, 0]
        t[i, 7:] = [np.float32(-0.1) + f * np.float32(0.05), np.float32(0.2) + f * np.float32(0.05),
                    np.float32(-0.3) + f * np.float32(0.05)]
        for ch in range(3):
            sh_cm[i, ch, 0] = np.float32(0.5) + f * np.float32(0.1)
            for j in range(1, coeffs):
                sh_cm[i, ch, j] = np.float32(j) * np.float32(0.1) + f * np.float32(0.01)
        o[i] = np.float32(0.8) - f * np.float32(0.1)
    # Splats::from_raw reads that flat list as [n, coeffs, 3]
    sh = sh_cm.reshape(n, coeffs, 3)
    return t, sh, o


@pytest.mark.parametrize("degree,rest_fields", [(0, 0), (1, 9), (2, 24), (3, 45)])
def test_header_field_counts(degree, rest_fields):
    text = checkpoint.ply_header(7, degree).decode()
    assert text.count("property float f_rest_") == rest_fields
    assert "f_dc_0" in text and "element vertex 7" in text and f"SH degree: {degree}" in text
    assert ("f_rest_0" in text) == (rest_fields > 0)
    assert f"f_rest_{rest_fields}" not in text
    assert text.endswith("end_header\n")


def test_header_metadata_round_trip():
    h = checkpoint.ply_header(0, 0, up_axis=(0.0, -1.0, 0.5), render_mode="mip")
    elements, comments, body, fmt = checkpoint._parse_header(h)
    assert fmt == "binary_little_endian" and body == len(h)
    assert elements[0].name == "vertex" and elements[0].count == 0 and len(elements[0].properties) == 14
    meta = checkpoint._metadata(comments, 0)
    assert meta.up_axis == (0.0, -1.0, 0.5) and meta.render_mode == "mip"
    assert "Vertical axis: 0 -1 0.5" in h.decode()
    m2 = checkpoint._metadata(["Vertical axis: z", "vertical axis: X", "SplatRenderMode: surfel"], 0)
    assert m2.up_axis == (1.0, 0.0, 0.0) and m2.render_mode == "surfel"
    assert checkpoint._metadata(["Vertical axis: y"], 0).up_axis == (0.0, -1.0, 0.0)


def test_oracle_rows_on_reference_test_splats():
    for degree in range(4):
        t, sh, o = reference_test_splats(degree, 5)
        rows = oracle.ply_encode(t, sh, o)
        coeffs, rest = (degree + 1) ** 2, (degree + 1) ** 2 - 1
        assert rows.shape == (5, 14 + 3 * rest)
        np.testing.assert_array_equal(rows[:, :3], t[:, :3])
        np.testing.assert_array_equal(rows[:, 3:6], t[:, 7:])
        np.testing.assert_array_equal(rows[:, 6], o)
        np.testing.assert_array_equal(rows[:, 7:11], t[:, 3:7])  # unit quaternions stay
        np.testing.assert_array_equal(rows[:, 11:14], sh[:, 0, :])
        for ch in range(3):  # rest coefficients channel-major
            np.testing.assert_array_equal(rows[:, 14 + ch * rest:14 + (ch + 1) * rest], sh[:, 1:, ch])
    t = np.zeros((3, 10), np.float32)
    t[0, 3:7] = [3, 4, 0, 0]
    t[2, 3:7] = [np.nan, 1, 0, 0]
    rows = oracle.ply_encode(t, np.zeros((3, 1, 3), np.float32), np.zeros(3, np.float32))
    np.testing.assert_array_equal(rows[0, 7:11], np.float32([0.6, 0.8, 0, 0]))
    np.testing.assert_array_equal(rows[1, 7:11], np.zeros(4, np.float32))  # |q| = 0 -> divided by 1e-12
    assert np.isnan(rows[2, 7]) and rows[2, 8] == np.float32(1e12)  # NaN norm -> 1e-12


def test_moment_dump_round_trip():
    optim = {"t": ops.Q8Moments(1000, "cpu"), "sh": ops.Q8Moments(4800, "cpu"), "o": ops.Q8Moments(100, "cpu"),
             "time": 1234}
    g = torch.Generator().manual_seed(0)
    for k in ("t", "sh", "o"):
        m = optim[k]
        m.m_codes.copy_(torch.randint(0, 256, m.m_codes.shape, generator=g, dtype=torch.uint8))
        m.v_codes.copy_(torch.randint(0, 256, m.v_codes.shape, generator=g, dtype=torch.uint8))
        m.m_scales.copy_(torch.rand(m.m_scales.shape, generator=g))
        m.v_scales.copy_(torch.rand(m.v_scales.shape, generator=g))
    buf = io.BytesIO()
    checkpoint.save_moments(buf, optim)
    buf.seek(0)
    back = checkpoint.load_moments(buf, "cpu")
    assert back["time"] == 1234
    for k in ("t", "sh", "o"):
        for a in ("m_codes", "v_codes", "m_scales", "v_scales"):
            assert torch.equal(getattr(back[k], a), getattr(optim[k], a)), (k, a)
    with pytest.raises(ValueError):
        checkpoint.load_moments(io.BytesIO(b"not a dump"), "cpu")


def test_header_rejects_other_layouts():
    with pytest.raises(ValueError):
        checkpoint._parse_header(b"obj\n")
