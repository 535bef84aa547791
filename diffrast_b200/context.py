"""Rasterization contexts: which device the ops run on (diffrast ``context.py``).

The class names, constructor arguments, attributes and error messages are diffrast's interface
(``RasterizeContext``, its nvdiffrast alias ``RasterizeCudaContext``, and ``RasterizeGLContext``,
whose ``output_db=False`` makes :func:`diffrast_b200.rasterize` return an empty
``[batch, height, width, 0]`` ``rast_db``). There is no OpenGL here: the GL context rasterizes
with the same CUDA kernels.
"""

from __future__ import annotations

import torch

DeviceSpec = torch.device | str | int | None


class RasterizeContext:
    """The device :func:`diffrast_b200.rasterize` runs on.

    Args:
        device: A ``torch.device``, a device string (``"cuda:1"``) or a GPU index. ``None`` means
            the current CUDA device, or the CPU when there is none (the ops then refuse to run).

    Attributes:
        device: The resolved device; a CUDA device always carries its index.
        output_db: Whether ``rast_db`` is returned. Always true for this class.
    """

    output_db = True

    def __init__(self, device: DeviceSpec = None) -> None:
        self.device = resolve_device(device)

    def __repr__(self) -> str:
        return f"{type(self).__name__}(device={str(self.device)!r})"

    def capture_overflowed(self) -> bool:
        """Whether a rasterization replayed from a CUDA graph on this device ran out of binning
        capacity since the last call (this synchronizes the device).

        A rasterization captured into a CUDA graph cannot read its binned-triangle counts back,
        so it bins into capacities taken from an eager call of the same shapes. A replay whose
        binned triangles exceed them sets a device word, and while that word is set every
        captured rasterization on the device is poisoned: the barycentrics, depth and ``rast_db``
        of its covered pixels are NaN, so the attributes, texture lookups, images and losses
        computed from them are NaN too. On ``True`` (which clears the word) the results of the
        replays since the last check are invalid; later captures get doubled capacities, so
        capture the graph again and rerun.
        """
        from diffrast_b200._kernels import capture_overflowed

        return capture_overflowed(self.device)


# nvdiffrast's name for the same context.
RasterizeCudaContext = RasterizeContext


class RasterizeGLContext(RasterizeContext):
    """nvdiffrast's OpenGL context, kept so that code creating one runs unchanged; it rasterizes
    exactly like :class:`RasterizeContext`.

    Args:
        output_db: ``False`` makes :func:`diffrast_b200.rasterize` return an empty
            ``[batch, height, width, 0]`` tensor in place of ``rast_db``.
        mode: Accepted and ignored.
        device: As for :class:`RasterizeContext`.
    """

    def __init__(self, output_db: bool = True, mode: str = "automatic",
                 device: DeviceSpec = None) -> None:
        # nvdiffrast takes the device first elsewhere; here a device in that place would read
        # as a true output_db, so it is refused.
        if isinstance(output_db, (str, torch.device)):
            raise TypeError(
                f"output_db must be a bool, got {output_db!r}; pass the device as device=..."
            )
        super().__init__(device)
        self.output_db = bool(output_db)
        self.mode = mode

    def __repr__(self) -> str:
        return f"RasterizeGLContext(output_db={self.output_db}, device={str(self.device)!r})"

    def set_context(self) -> None:
        """No-op: no OpenGL context exists."""

    def release_context(self) -> None:
        """No-op: no OpenGL context exists."""


def _as_device(spec: DeviceSpec) -> torch.device:
    """``spec`` as a ``torch.device`` (index not yet filled in)."""
    if spec is None:
        return torch.device("cuda" if torch.cuda.is_available() else "cpu")
    if isinstance(spec, (torch.device, str)):
        return torch.device(spec)
    index = getattr(type(spec), "__index__", None)
    if index is None or isinstance(spec, bool):
        raise TypeError(
            f"device must be a torch.device, a string or a GPU index, got {spec!r}."
        )
    gpu = index(spec)
    if gpu < 0:
        raise ValueError(f"device must not be a negative GPU index, got {spec!r}.")
    return torch.device("cuda", gpu)


def resolve_device(spec: DeviceSpec) -> torch.device:
    """The device a context runs on: ``spec`` resolved, with the index of a CUDA device filled in
    and checked against the devices present."""
    device = _as_device(spec)
    if device.type != "cuda":
        return device
    available = torch.cuda.device_count() if torch.cuda.is_available() else 0
    if available == 0:
        raise RuntimeError(
            f"device {str(device)!r} was requested, but no CUDA or ROCm device is available."
        )
    index = torch.cuda.current_device() if device.index is None else device.index
    if index >= available:
        raise ValueError(
            f"device {str(device)!r} does not exist; {available} CUDA or ROCm "
            "devices are available."
        )
    return torch.device("cuda", index)
