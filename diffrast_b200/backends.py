"""Backend selection kept as API surface (diffrast backends/__init__.py:18-52).

diffrast_b200 has exactly one backend, the CUDA kernels of ``libdiffrast_b200.so``, and no
multi-backend dispatch or CPU fallback. ``set_backend`` accepts the names the reference accepts
so that code calling it keeps running; every op runs on the CUDA backend regardless.
"""

from __future__ import annotations

import torch

BACKENDS = ("cuda",)
OPS = ("rasterize", "interpolate", "texture", "antialias")
_ACCEPTED = ("auto", "cuda", "triton", "reference")
_selected = "auto"


def set_backend(name: str) -> None:
    """Accepts ``"auto"``, ``"cuda"``, ``"triton"`` or ``"reference"``; all select the CUDA kernels."""
    global _selected
    if name not in _ACCEPTED:
        options = ", ".join(repr(n) for n in _ACCEPTED)
        raise ValueError(f"Unknown backend {name!r}; expected one of {options}.")
    _selected = name


def get_backend_name(device: torch.device | str, op: str) -> str:
    """Name of the backend ``op`` runs on for tensors on ``device``: always ``"cuda"``."""
    if op not in OPS:
        raise ValueError(f"Unknown op {op!r}; expected one of {OPS}.")
    require_cuda(torch.device(device))
    return "cuda"


def require_cuda(device: torch.device) -> None:
    if device.type != "cuda":
        raise RuntimeError(
            "diffrast_b200 runs on CUDA devices only (B200, sm_100a) and has no CPU fallback; "
            f"got tensors on {str(device)!r}."
        )
