"""Rasterization contexts (diffrast context.py:8-102): the device the ops run on."""

from __future__ import annotations

import operator

import torch


class RasterizeContext:
    """Device that :func:`diffrast_b200.rasterize` runs on.

    Args:
        device: A ``torch.device``, a string such as ``"cuda:0"`` or a GPU index. Defaults to the
            current CUDA device (the CPU when none is available; the ops then refuse to run).

    Attributes:
        device: The resolved device, with an explicit index for a GPU.
        output_db: Whether :func:`diffrast_b200.rasterize` returns ``rast_db``; always true here.
    """

    output_db = True

    def __init__(self, device: torch.device | str | int | None = None) -> None:
        self.device = _resolve_device(device)

    def __repr__(self) -> str:
        return f"{type(self).__name__}(device={str(self.device)!r})"

    def capture_overflowed(self) -> bool:
        """Whether a rasterization replayed from a CUDA graph on this device ran out of binning
        capacity since the last call (this synchronizes the device).

        A call captured into a CUDA graph cannot read its binned-triangle counts back, so it uses
        capacities measured by an eager call of the same shapes (twice the counts seen). Triangles
        whose pixel box exceeds 512 pixels beyond that capacity are then missing from the result.
        On ``True`` the results of the replays since the last check are incomplete; the
        capacities of later captures are doubled, so capture the graph again and rerun.
        """
        from diffrast_b200._kernels import capture_overflowed

        return capture_overflowed(self.device)


# nvdiffrast's name for the same context.
RasterizeCudaContext = RasterizeContext


class RasterizeGLContext(RasterizeContext):
    """Stand-in for nvdiffrast's OpenGL context: rasterizes exactly like :class:`RasterizeContext`.

    Args:
        output_db: Whether ``rast_db`` is returned; with ``False`` an empty
            ``[batch, height, width, 0]`` tensor takes its place.
        mode: Accepted for compatibility and ignored.
        device: As for :class:`RasterizeContext`.
    """

    def __init__(self, output_db: bool = True, mode: str = "automatic",
                 device: torch.device | str | int | None = None) -> None:
        super().__init__(device)
        if isinstance(output_db, (str, torch.device)):
            raise TypeError(
                f"output_db must be a bool, got {output_db!r}; pass the device as device=..."
            )
        self.output_db = bool(output_db)
        self.mode = mode

    def __repr__(self) -> str:
        return f"RasterizeGLContext(output_db={self.output_db}, device={str(self.device)!r})"

    def set_context(self) -> None:
        """Nothing to do: there is no OpenGL context."""

    def release_context(self) -> None:
        """Nothing to do: there is no OpenGL context."""


def _resolve_device(device) -> torch.device:
    if device is None:
        device = "cuda" if torch.cuda.is_available() else "cpu"
    elif not isinstance(device, (torch.device, str)):
        try:
            if isinstance(device, bool):
                raise TypeError
            index = operator.index(device)
        except TypeError:
            raise TypeError(
                f"device must be a torch.device, a string or a GPU index, got {device!r}."
            ) from None
        if index < 0:
            raise ValueError(f"device must not be a negative GPU index, got {device!r}.")
        device = torch.device("cuda", index)
    device = torch.device(device)
    if device.type != "cuda":
        return device
    if not torch.cuda.is_available():
        raise RuntimeError(
            f"device {str(device)!r} was requested, but no CUDA or ROCm device is available."
        )
    if device.index is None:
        return torch.device("cuda", torch.cuda.current_device())
    if device.index >= torch.cuda.device_count():
        raise ValueError(
            f"device {str(device)!r} does not exist; {torch.cuda.device_count()} CUDA or ROCm "
            "devices are available."
        )
    return device
