"""ctypes binding of ``libdiffrast_b200.so``, the C ABI declared in ``include/diffrast_b200.h``.

The library is loaded from ``diffrast_b200/_lib``; there is no fallback: if it is missing the
first op raises ``ImportError`` with the command that builds it. Every entry point returns a status
that :func:`check` turns into a ``RuntimeError`` naming the call.
"""

from __future__ import annotations

import ctypes
import os
import threading
from ctypes import POINTER, c_char_p, c_float, c_int, c_int32, c_int64, c_size_t, c_void_p
from pathlib import Path

import torch

LIBDIR = Path(__file__).resolve().parent / "_lib"
# DIFFRAST_B200_CHECK=1 loads the checked build: every index read from the data (tri, rast ids,
# keys, opposite vertices, attribute rows, texel offsets) is bounds-checked on the device, and
# every call synchronizes and raises on the first recorded fault (slow; for debugging).
CHECKED = os.environ.get("DIFFRAST_B200_CHECK", "0") not in ("", "0")
LIBRARY = LIBDIR / ("libdiffrast_b200_checked.so" if CHECKED else "libdiffrast_b200.so")

FILTER_MODES = ("nearest", "linear", "linear-mipmap-nearest", "linear-mipmap-linear")
BOUNDARY_MODES = ("wrap", "clamp", "zero", "cube")
MAX_LEVELS = 32

_P = c_void_p
_SIGNATURES = {
    "dr_version": (c_int, []),
    "dr_status_string": (c_char_p, [c_int]),
    "dr_raster_setup_workspace_bytes": (c_size_t, [c_int64, c_int32, c_int32]),
    "dr_raster_setup": (
        c_int,
        [_P, c_int64, _P, c_int64, c_int64, c_int64, _P, _P, c_int64, c_int32, c_int32, _P, _P, _P,
         c_size_t, c_int64, _P, c_size_t, _P],
    ),
    "dr_raster_occlusion_workspace_bytes": (c_size_t, [c_int64, c_int64, c_int32, c_int32]),
    "dr_raster_occluded": (
        c_int,
        [_P, c_int64, _P, c_int64, c_int64, c_int64, _P, _P, c_int64, c_int32, c_int32, _P, _P, _P,
         _P, c_size_t, _P],
    ),
    "dr_raster_counts": (c_int, [_P, POINTER(c_int64), POINTER(c_int64), _P]),
    "dr_raster_bin_workspace_bytes": (c_size_t, [c_int64, c_int32, c_int32, c_int64]),
    "dr_raster_tiles": (
        c_int,
        [_P, c_int64, _P, c_int64, c_int64, c_int64, c_int32, c_int32, _P, _P, _P, c_int64,
         c_int64, _P, c_size_t, _P],
    ),
    "dr_raster_tiles_device": (
        c_int,
        [_P, c_int64, _P, c_int64, c_int64, c_int64, c_int32, c_int32, _P, _P, _P, c_int64,
         c_int64, _P, c_size_t, _P, _P],
    ),
    "dr_raster_poison_keys": (c_int, [_P, _P, c_int64, _P]),
    "dr_raster_resolve_fwd": (
        c_int, [_P, c_int64, _P, _P, c_int64, c_int64, c_int64, c_int32, c_int32, _P, _P, _P]
    ),
    "dr_raster_resolve_bwd": (
        c_int, [_P, c_int64, _P, _P, c_int64, c_int64, c_int64, c_int32, c_int32, _P, _P, _P, _P]
    ),
    "dr_interpolate_fwd": (
        c_int,
        [_P, c_int64, c_int64, c_int32, c_int32, _P, _P, _P, c_int64, _P, c_int32, c_int64,
         c_int32, c_int32, _P, _P, _P],
    ),
    "dr_interpolate_bwd": (
        c_int,
        [_P, c_int64, c_int64, c_int32, _P, _P, _P, c_int64, _P, c_int32, c_int64, c_int32,
         c_int32, _P, _P, _P, _P, _P, _P],
    ),
    "dr_interpolate_bwd_parts": (
        c_int,
        [_P, c_int64, c_int64, c_int32, _P, _P, _P, c_int64, _P, c_int32, c_int64, c_int32,
         c_int32, _P, _P, _P, c_int32, c_int32, _P, c_int32, c_int32, _P, _P, _P, _P],
    ),
    "dr_texture_fwd": (
        c_int,
        [_P, _P, _P, _P, c_int32, c_int32, _P, c_int64, _P, c_int64, _P, c_int64, c_int32,
         c_int32, c_int32, c_int32, _P, _P],
    ),
    "dr_texture_bwd": (
        c_int,
        [_P, _P, _P, _P, _P, c_int32, c_int32, c_int32, _P, c_int64, _P, c_int64, _P, c_int64,
         c_int32, c_int32, c_int32, c_int32, _P, _P, c_int64, c_int32, _P, c_int64, c_int32, _P,
         _P],
    ),
    "dr_texture_bwd_interp": (
        c_int,
        [_P, _P, _P, _P, _P, c_int32, c_int32, c_int32, _P, c_int64, _P, c_int64, _P, c_int64,
         c_int32, c_int32, c_int32, c_int32, _P, _P, _P, _P, c_int64, _P, c_int64, c_int64,
         c_int32, c_int32, c_int32, c_int32, c_int32, _P, _P, _P],
    ),
    "dr_texture_bwd_resolve": (
        c_int,
        [_P, _P, _P, _P, _P, c_int32, c_int32, c_int32, _P, c_int64, _P, c_int64, _P, c_int64,
         c_int32, c_int32, c_int32, c_int32, _P, _P, _P, _P, c_int64, _P, c_int64, c_int64,
         c_int32, c_int32, c_int32, c_int32, c_int32, _P, _P, c_int64, c_int64, c_int32, _P, _P],
    ),
    "dr_texture_chain_bwd": (
        c_int,
        [_P, _P, c_int64, c_int32, c_int32, _P, c_int64, _P, c_int64, c_int64, c_int32, c_int32,
         c_int32, c_int32, c_int32, _P, _P, c_int64, c_int64, c_int32, _P, _P],
    ),
    "dr_mip_downsample": (c_int, [_P, c_int64, c_int32, c_int32, c_int32, _P, _P]),
    "dr_mip_build": (c_int, [_P, c_int64, c_int32, c_int32, c_int32, c_int32, _P, _P]),
    "dr_mip_build_bwd": (c_int, [_P, c_int64, c_int32, c_int32, c_int32, c_int32, _P, c_int32, _P]),
    "dr_mip_downsample_bwd": (c_int, [_P, c_int64, c_int32, c_int32, c_int32, _P, _P, c_int32, _P]),
    "dr_edge_neighbours_workspace_bytes": (c_size_t, [c_int64]),
    "dr_edge_neighbours": (c_int, [_P, c_int64, _P, _P, c_size_t, _P]),
    "dr_edge_neighbours_noalloc_max_triangles": (c_int64, []),
    "dr_edge_neighbours_noalloc": (c_int, [_P, c_int64, _P, _P]),
    "dr_edge_opposite_vertices": (c_int, [_P, _P, c_int64, _P, _P]),
    "dr_silhouette_edges": (c_int, [_P, c_int64, c_int64, _P, c_int64, _P, _P, _P]),
    "dr_antialias_pair_bytes": (c_size_t, [c_int64, c_int32, c_int32]),
    "dr_antialias_fwd": (
        c_int,
        [_P, _P, _P, c_int64, c_int64, _P, c_int64, _P, c_int64, c_int32, c_int32, c_int32, _P,
         _P, c_size_t, _P],
    ),
    "dr_antialias_bwd": (
        c_int,
        [_P, _P, _P, c_int64, c_int64, _P, c_int64, _P, c_int64, c_int32, c_int32, c_int32, _P,
         c_float, _P, c_size_t, _P, _P, _P],
    ),
    "dr_antialias_loss_partials": (c_size_t, [c_int64, c_int32, c_int32]),
    "dr_antialias_mse_fwd": (
        c_int,
        [_P, _P, _P, c_int64, c_int64, _P, c_int64, _P, c_int64, c_int32, c_int32, c_int32, _P,
         _P, _P, _P, c_size_t, _P, c_size_t, _P],
    ),
    "dr_antialias_mse_bwd": (
        c_int,
        [_P, _P, _P, c_int64, c_int64, _P, c_int64, _P, c_int64, c_int32, c_int32, c_int32, _P,
         _P, c_float, _P, c_float, _P, c_size_t, _P, _P, _P],
    ),
    "dr_lambert_fwd": (
        c_int, [_P, _P, c_int64, _P, c_int64, c_float, c_int64, c_int32, c_int32, c_int32, _P, _P]
    ),
    "dr_lambert_bwd": (
        c_int,
        [_P, _P, c_int64, _P, c_int64, c_float, c_int64, c_int32, c_int32, c_int32, _P, _P, _P,
         _P],
    ),
    "dr_zero": (c_int, [_P, c_size_t, _P]),
    "dr_checked_build": (c_int, []),
    "dr_check_faults": (c_int, [POINTER(ctypes.c_uint64)]),
    "dr_check_site_name": (c_char_p, [c_int]),
    "dr_to_clip_fwd": (c_int, [_P, c_int64, _P, c_int64, _P, _P]),
    "dr_to_clip_bwd": (c_int, [_P, _P, c_int64, _P, c_int64, _P, _P, _P]),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def symbols() -> list[str]:
    """Names of every C-ABI entry point this binding uses."""
    return list(_SIGNATURES)


def lib() -> ctypes.CDLL:
    """The loaded library (loaded on first use)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIBRARY.exists():
                how = " --checked" if CHECKED else ""
                raise ImportError(
                    f"{LIBRARY} is missing; build it with `python -m diffrast_b200.build{how}` "
                    "(needs nvcc). diffrast_b200 has no CPU fallback."
                )
            handle = ctypes.CDLL(str(LIBRARY))
            for name, (restype, argtypes) in _SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = restype
                fn.argtypes = argtypes
            _lib = handle
    return _lib


def check(status: int, call: str) -> None:
    if status != 0:
        message = lib().dr_status_string(status).decode()
        raise RuntimeError(f"diffrast_b200: {call} failed with status {status}: {message}")
    if CHECKED:
        check_faults(call)


class BoundsFault(RuntimeError):
    """A bounds check of the checked build failed: ``site`` names the kind of index, ``index``
    its value (the low 48 bits)."""

    def __init__(self, call: str, site: str, index: int) -> None:
        super().__init__(f"diffrast_b200: {call}: out-of-bounds {site}: {index}")
        self.site = site
        self.index = index


def check_faults(call: str = "a kernel") -> None:
    """Raise :class:`BoundsFault` if a checked-build kernel recorded an out-of-bounds index since
    the last check (synchronizes the device; a no-op for the ordinary build)."""
    fault = ctypes.c_uint64(0)
    status = lib().dr_check_faults(ctypes.byref(fault))
    if status != 0:
        message = lib().dr_status_string(status).decode()
        raise RuntimeError(f"diffrast_b200: dr_check_faults failed with status {status}: {message}")
    if fault.value:
        site = lib().dr_check_site_name(fault.value >> 48).decode()
        index = fault.value & 0xFFFFFFFFFFFF
        if index >= 1 << 47:
            index -= 1 << 48  # negative indices come back sign-extended
        raise BoundsFault(call, site, index)


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def int32_array(values) -> ctypes.Array:
    return (c_int32 * len(values))(*values)


def int64_array(values) -> ctypes.Array:
    return (c_int64 * len(values))(*values)


def pointer_array(values) -> ctypes.Array:
    return (c_void_p * len(values))(*values)
