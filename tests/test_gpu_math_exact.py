"""The kernels replace IEEE sqrtf and 1/x by cheaper fma-refined sequences
(sqrt_rn, rcp_rn in vs_common.cuh) on the claim that they are correctly
rounded.  These tests check that claim on the device for every input it is
made for: all non-negative floats for the square root, and every b with
|b| in [2^-126, 2^126) for the reciprocal (both signs)."""
import pytest
import torch

from vauss_b200 import ops

pytestmark = pytest.mark.gpu

CHUNK = 1 << 27


def _all_bits(cuda, lo, hi):
    for start in range(lo, hi, CHUNK):
        stop = min(start + CHUNK, hi)
        yield torch.arange(start, stop, dtype=torch.int64, device=cuda).to(torch.int32).view(torch.float32)


def _mismatches(got, want):
    g, w = got.view(torch.int32), want.view(torch.int32)
    both_nan = torch.isnan(got) & torch.isnan(want)
    return int(((g != w) & ~both_nan).sum())


def test_sqrt_rn_matches_ieee_for_every_nonnegative_float(cuda):
    bad = 0
    for x in _all_bits(cuda, 0, 0x7F800001):  # +0 ... +inf
        bad += _mismatches(ops.math_probe("sqrt_rn", x), ops.math_probe("sqrt_ieee", x))
    assert bad == 0


def test_rcp_rn_matches_ieee_over_its_range(cuda):
    bad = 0
    for x in _all_bits(cuda, 0x00800000, 0x7E800000):  # [2^-126, 2^126)
        bad += _mismatches(ops.math_probe("rcp_rn", x), ops.math_probe("rcp_ieee", x))
        xn = -x
        bad += _mismatches(ops.math_probe("rcp_rn", xn), ops.math_probe("rcp_ieee", xn))
    assert bad == 0
