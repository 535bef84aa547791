"""The bounds-checked build (DIFFRAST_B200_CHECK=1): on the CPU, that it loads, exports every
entry point of the header and reports itself as checked while the ordinary build does not."""

import ctypes
import subprocess
import sys
from pathlib import Path

from diffrast_b200 import _native

ROOT = Path(__file__).resolve().parents[1]


def test_checked_library_loads_and_exports_every_entry_point():
    checked = _native.LIBDIR / "libdiffrast_b200_checked.so"
    ordinary = _native.LIBDIR / "libdiffrast_b200.so"
    for path, flag in ((checked, 1), (ordinary, 0)):
        handle = ctypes.CDLL(str(path))
        for name in _native.symbols():
            assert hasattr(handle, name), (path.name, name)
        assert handle.dr_checked_build() == flag
        handle.dr_check_site_name.restype = ctypes.c_char_p
        assert handle.dr_check_site_name(2).decode() == "vertex index read from tri"


def test_environment_variable_selects_the_checked_library():
    code = ("from diffrast_b200 import _native; "
            "print(_native.LIBRARY.name, _native.lib().dr_checked_build())")
    for value, expected in (("1", "libdiffrast_b200_checked.so 1"), ("0", "libdiffrast_b200.so 0")):
        out = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True,
                             text=True, check=True, env={"DIFFRAST_B200_CHECK": value,
                                                         "PATH": "/usr/bin:/bin"})
        assert out.stdout.split() == expected.split()
