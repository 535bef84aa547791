"""Edge adjacency of an index buffer: the part of silhouette detection that depends only on
``tri`` (diffrast ``topology.py``; format of ``reference.py:768-787``).

The antialias kernels need, for every triangle edge, the vertex across it in the neighbouring
triangle. Both tables are built on the GPU in one pass over a hash table of vertex-pair keys
(``dr_edge_neighbours``, then ``dr_edge_opposite``), once per index buffer: explicitly with
``antialias_construct_topology_hash``, or through a per-tensor cache keyed on the ``tri`` object.
"""

from __future__ import annotations

import weakref

import torch
from torch import Tensor

from diffrast_b200._cache import TensorCache, signature
from diffrast_b200.backends import require_cuda


def edge_neighbours(tri: Tensor) -> Tensor:
    """For edge ``3 t + k`` (opposite vertex ``k``) the edge sharing its vertex pair, or -1 when
    none or several do; int64 ``[triangles, 3]`` on ``tri``'s device."""
    from diffrast_b200 import _kernels as K

    require_cuda(tri.device)
    with torch.cuda.device(tri.device):
        return K.edge_neighbours(tri.contiguous())


class _Provenance:
    """Which tensor object a topology was built from, and its signature then: enough to tell that
    the very same tensor was edited in place afterwards. It is not copied or pickled with the
    topology (a weak reference cannot be), so copies only check shape and device."""

    __slots__ = ("source", "sig")

    def __init__(self, tri: Tensor) -> None:
        self.source = weakref.ref(tri)
        self.sig = signature(tri)

    def edited(self, tri: Tensor) -> bool:
        return self.source() is tri and signature(tri) != self.sig


class TopologyHash:
    """Edge adjacency of an index buffer, as built by ``antialias_construct_topology_hash``.

    Pass it to :func:`diffrast_b200.antialias` with the ``tri`` it was built from, or a tensor of
    the same shape and contents on the same device.
    """

    def __init__(self, tri: Tensor) -> None:
        from diffrast_b200 import _kernels as K

        neighbours = edge_neighbours(tri)
        with torch.cuda.device(tri.device):
            # The vertex across each edge (-1: a silhouette by topology alone).
            opposite = K.edge_opposite(tri.contiguous(), neighbours)
        self._init_tables(neighbours, opposite, tuple(tri.shape), tri.device, _Provenance(tri))

    def _init_tables(self, neighbours, opposite, shape, device, provenance) -> None:
        self._neighbours = neighbours
        self._opposite = opposite
        self._shape = shape
        self._device = device
        self._provenance = provenance

    @classmethod
    def _from_tables(cls, neighbours, opposite, shape, device) -> TopologyHash:
        topo = cls.__new__(cls)
        topo._init_tables(neighbours, opposite, shape, device, None)
        return topo

    def __reduce__(self):
        # Copies and pickles carry the tables; the provenance link stays with the original.
        return (TopologyHash._from_tables,
                (self._neighbours, self._opposite, self._shape, self._device))

    def __repr__(self) -> str:
        return f"TopologyHash(triangles={self._shape[0]}, device={str(self._device)!r})"

    def neighbours(self, tri: Tensor) -> Tensor:
        """The adjacency, int64 ``[triangles, 3]``, after checking that it can belong to ``tri``."""
        self.validate(tri)
        return self._neighbours

    def opposite(self, tri: Tensor) -> Tensor:
        """For edge ``3 t + k`` the vertex opposite it in the adjacent triangle, -1 without one;
        int32 ``[triangles, 3]``, after checking that it can belong to ``tri``."""
        self.validate(tri)
        return self._opposite

    def validate(self, tri: Tensor) -> None:
        """Raise ``ValueError`` unless this topology can belong to ``tri``."""
        shape = tuple(tri.shape)
        if shape != self._shape or tri.device != self._device:
            raise ValueError(
                f"topology_hash was built for a tri of shape {self._shape} on {self._device}, "
                f"got shape {shape} on {tri.device}."
            )
        if self._provenance is not None and self._provenance.edited(tri):
            raise ValueError(
                "tri was modified in place after topology_hash was built from it; build a new "
                "one with antialias_construct_topology_hash."
            )


# An entry holds 20 bytes per triangle on the GPU (int64 neighbours, int32 opposite vertices),
# so only a few index buffers are remembered.
_cached_topologies: TensorCache[TopologyHash] = TensorCache(TopologyHash, max_entries=16)


def topology_for(tri: Tensor, topology_hash: TopologyHash | None) -> TopologyHash:
    """``topology_hash`` after checking it against ``tri``; without one, ``tri``'s cached
    topology (built on first use)."""
    if topology_hash is None:
        return _cached_topologies.get(tri)
    if isinstance(topology_hash, TopologyHash):
        topology_hash.validate(tri)
        return topology_hash
    raise TypeError(
        "topology_hash must come from antialias_construct_topology_hash, got "
        f"{type(topology_hash).__name__}."
    )
