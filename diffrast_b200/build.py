"""Build the CUDA library of diffrast_b200 for B200 (sm_100a) in the source tree.

``python -m diffrast_b200.build`` (or :func:`build`) compiles every ``csrc/*.cu`` with nvcc for
``sm_100a`` and links ``diffrast_b200/_lib/libdiffrast_b200.so``, a plain C-ABI shared library
(see ``include/diffrast_b200.h``) with the CUDA runtime linked statically. Objects are rebuilt
only when a source or header is newer. The build needs nvcc but no GPU.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
ROOT = PACKAGE.parent
CSRC = PACKAGE / "csrc"
BUILD = PACKAGE / "_build"
LIBDIR = PACKAGE / "_lib"
LIBRARY = LIBDIR / "libdiffrast_b200.so"
# The checked build (every data-dependent index bounds-checked, faults recorded instead of taken;
# loaded with DIFFRAST_B200_CHECK=1).
CHECKED_LIBRARY = LIBDIR / "libdiffrast_b200_checked.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC,-O3",
    f"-I{ROOT / 'include'}",
]


def nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(found).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is needed to build diffrast_b200")
    return found


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(verbose: bool = False, ptxas_verbose: bool = False, checked: bool = False) -> Path:
    """Compile and link the library (the checked variant with ``checked``); returns its path."""
    build_dir = BUILD / "checked" if checked else BUILD
    library = CHECKED_LIBRARY if checked else LIBRARY
    build_dir.mkdir(parents=True, exist_ok=True)
    LIBDIR.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    headers = sorted(CSRC.glob("*.cuh")) + sorted((ROOT / "include").glob("*.h"))
    compiler = nvcc()
    extra = ["-Xptxas", "-v"] if ptxas_verbose else []
    if checked:
        extra.append("-DDR_CHECKED=1")

    def compile_one(src: Path) -> tuple[Path, str]:
        obj = build_dir / (src.stem + ".o")
        if ptxas_verbose or _stale(obj, [src, *headers, Path(__file__)]):
            cmd = [compiler, *ARCH, *FLAGS, *extra, "-c", str(src), "-o", str(obj)]
            res = subprocess.run(cmd, capture_output=True, text=True)
            if res.returncode != 0:
                raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
            return obj, res.stdout + res.stderr
        return obj, ""

    workers = max(1, min(len(sources), os.cpu_count() or 1))
    with ThreadPoolExecutor(workers) as pool:
        results = list(pool.map(compile_one, sources))
    objects = [obj for obj, _ in results]
    if verbose or ptxas_verbose:
        for _, log in results:
            if log:
                print(log, file=sys.stderr)
    if _stale(library, objects):
        tmp = library.with_suffix(".so.tmp")
        cmd = [compiler, *ARCH, "-shared", "-cudart", "static", *map(str, objects), "-o", str(tmp)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"linking failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, library)
    return library


if __name__ == "__main__":
    print(build(verbose=True, ptxas_verbose="-v" in sys.argv, checked="--checked" in sys.argv))
