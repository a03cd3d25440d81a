"""The C-ABI library loads and exports every entry point include/*.h declares
(no compute calls: no GPU here)."""
import glob
import os
import re

from tests.conftest import ROOT


def _declared():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        names |= set(re.findall(r"VS_API\s+[\w\s\*]+?\b(vs_\w+)\s*\(", src))
    return names


def test_header_declares_entry_points():
    names = _declared()
    for must in ("vs_render_forward", "vs_loss", "vs_rasterize_backward", "vs_project_update", "vs_sh_step",
                 "vs_step_q8", "vs_vjp_dense", "vs_adam_q8_dense", "vs_gather_stats", "vs_noise_means"):
        assert must in names


def test_library_exports_every_declared_symbol(native_lib):
    missing = [n for n in sorted(_declared()) if not hasattr(native_lib, n)]
    assert not missing, f"exported symbols missing: {missing}"


def test_binding_covers_header(native_lib):
    from vauss_b200 import _native
    assert set(_native.EXPORTED) == _declared()


def test_version_string(native_lib):
    assert b"sm_100a" in native_lib.vs_version()
