"""Depth peeling (diffrast peeling.py:12-92): successive depth layers of the same geometry.

The per-pixel state between layers is the packed 64-bit visibility key of the previous layer,
kept on the device; each layer rasterizes only keys ordered after it.
"""

from __future__ import annotations

from types import TracebackType

from torch import Tensor

from diffrast_b200.context import RasterizeContext
from diffrast_b200 import _kernels as K
from diffrast_b200.ops import check_rasterize_inputs, rasterize_layer


class DepthPeeler:
    """Rasterize successive depth layers; the first equals :func:`rasterize`.

    Each later layer gives, per pixel, the nearest triangle behind the previous one, ordered by
    depth and then by index. The peeler keeps copies of ``pos``, ``tri`` and ``ranges`` (gradients
    still reach the ``pos`` passed in). Used as a context manager, it is closed on exit::

        with DepthPeeler(glctx, pos, tri, (512, 512)) as peeler:
            for _ in range(num_layers):
                rast, rast_db = peeler.rasterize_next_layer()
    """

    def __init__(self, glctx: RasterizeContext, pos: Tensor, tri: Tensor,
                 resolution: tuple[int, int], ranges: Tensor | None = None,
                 grad_db: bool = True) -> None:
        self._resolution = check_rasterize_inputs(glctx, pos, tri, resolution, ranges)
        self._output_db = getattr(glctx, "output_db", True)
        self._grad_db = grad_db and self._output_db
        self._pos, self._tri = pos.clone(), tri.clone()
        self._ranges = K.range_table(ranges, pos.device) if pos.ndim == 2 else None
        self._state = None
        self._closed = False

    def __enter__(self) -> DepthPeeler:
        return self

    def __exit__(self, exc_type: type[BaseException] | None, exc_value: BaseException | None,
                 traceback: TracebackType | None) -> None:
        self._state = None
        self._closed = True

    def rasterize_next_layer(self) -> tuple[Tensor, Tensor]:
        """``(rast, rast_db)`` of the next depth layer."""
        if self._closed:
            raise RuntimeError(
                "This DepthPeeler was closed when its with block exited; create a new one to "
                "rasterize more layers."
            )
        rast, rast_db, self._state = rasterize_layer(
            self._pos, self._tri, self._resolution, self._grad_db, self._state, self._ranges
        )
        return rast, (rast_db if self._output_db else rast.new_zeros(*rast.shape[:3], 0))
