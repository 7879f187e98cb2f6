"""CPU-only checks of the C-ABI library: it builds for sm_100a, loads without a GPU, and exports every
function that include/osam.h declares (no compute calls — there is no device here)."""
import ctypes
import subprocess

from objectsam_b200 import _lib, build


def test_library_builds_and_exports_every_header_symbol():
    path = build.build()
    names = _lib.header_symbols()
    assert "osam_conv_fwd" in names and "osam_conv_plan_create" in names
    so = ctypes.CDLL(path)
    missing = [n for n in names if not hasattr(so, n)]
    assert not missing, f"symbols declared in include/osam.h but not exported: {missing}"
    out = subprocess.run(["nm", "-D", "--defined-only", path], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert set(names) <= exported


def test_binding_covers_header():
    assert set(_lib.header_symbols()) == set(_lib._SIGS), "ctypes signatures out of sync with include/osam.h"

