"""The C ABI from a plain C program: the header compiles as C (gcc, -std=c99 -Wall -Werror) and a
binary linked against the library calls it, without Python and without a GPU (only calls that
fail validation are made)."""

import shutil
import subprocess
from pathlib import Path

import pytest

from diffrast_b200 import _native

ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_header_compiles_as_c_and_entry_points_are_callable(tmp_path):
    lib = Path(_native.LIBRARY)
    exe = tmp_path / "c_abi_check"
    subprocess.run(
        ["gcc", "-std=c99", "-Wall", "-Werror", f"-I{ROOT / 'include'}",
         str(ROOT / "tests" / "c_abi_check.c"), str(lib), f"-Wl,-rpath,{lib.parent}", "-o",
         str(exe)],
        check=True, capture_output=True, text=True,
    )
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, (out.returncode, out.stdout, out.stderr)
    assert "c abi ok: workspace too small" in out.stdout
