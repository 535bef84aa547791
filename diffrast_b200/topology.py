"""Edge adjacency of an index buffer, the ``tri``-only part of silhouette detection
(diffrast topology.py:19-72).

The adjacency is built on the GPU by ``dr_edge_neighbours`` (a hash table on vertex-pair keys),
once per index buffer: explicitly through ``antialias_construct_topology_hash`` or through a cache
keyed on the ``tri`` tensor object.
"""

from __future__ import annotations

import weakref

import torch
from torch import Tensor

from diffrast_b200._cache import TensorCache, stamp
from diffrast_b200.backends import require_cuda


def edge_neighbours(tri: Tensor) -> Tensor:
    """For edge ``3 t + k`` (opposite vertex ``k``) the edge sharing its vertex pair, or -1 when
    none or several do; int64 ``[triangles, 3]`` on ``tri``'s device."""
    from diffrast_b200 import _kernels as K

    require_cuda(tri.device)
    with torch.cuda.device(tri.device):
        return K.edge_neighbours(tri.contiguous())


class TopologyHash:
    """Edge adjacency of an index buffer, as built by ``antialias_construct_topology_hash``.

    Pass it to :func:`diffrast_b200.antialias` with the ``tri`` it was built from, or a tensor of
    the same shape and contents on the same device.
    """

    def __init__(self, tri: Tensor) -> None:
        from diffrast_b200 import _kernels as K

        self._neighbours = edge_neighbours(tri)
        with torch.cuda.device(tri.device):
            # The kernels' form: the vertex across each edge (-1: silhouette by topology).
            self._opposite = K.edge_opposite(tri.contiguous(), self._neighbours)
        self._shape = tuple(tri.shape)
        self._device = tri.device
        self._source: weakref.ref | None = weakref.ref(tri)
        self._stamp = stamp(tri)

    def __repr__(self) -> str:
        return f"TopologyHash(triangles={self._shape[0]}, device={str(self._device)!r})"

    def __getstate__(self) -> dict:
        # Copies keep the adjacency but not the link used to notice in-place edits.
        return {**self.__dict__, "_source": None, "_stamp": None}

    def neighbours(self, tri: Tensor) -> Tensor:
        self._check(tri)
        return self._neighbours

    def opposite(self, tri: Tensor) -> Tensor:
        """For edge ``3 t + k`` the vertex opposite it in the adjacent triangle, -1 without one;
        int32 ``[triangles, 3]``."""
        self._check(tri)
        return self._opposite

    def _check(self, tri: Tensor) -> None:
        if tuple(tri.shape) != self._shape or tri.device != self._device:
            raise ValueError(
                f"topology_hash was built for a tri of shape {self._shape} on {self._device}, "
                f"got shape {tuple(tri.shape)} on {tri.device}."
            )
        if self._source is not None and self._source() is tri and stamp(tri) != self._stamp:
            raise ValueError(
                "tri was modified in place after topology_hash was built from it; build a new "
                "one with antialias_construct_topology_hash."
            )


# Each entry holds three times the size of its index buffer, so only a few are kept.
_topology_cache: TensorCache[TopologyHash] = TensorCache(TopologyHash, max_entries=16)


def topology_for(tri: Tensor, topology_hash: TopologyHash | None) -> TopologyHash:
    """``topology_hash`` if given (checked), else the cached adjacency of ``tri``."""
    if topology_hash is None:
        return _topology_cache.get(tri)
    if not isinstance(topology_hash, TopologyHash):
        raise TypeError(
            "topology_hash must come from antialias_construct_topology_hash, got "
            f"{type(topology_hash).__name__}."
        )
    topology_hash._check(tri)
    return topology_hash
