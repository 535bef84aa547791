"""Per-tensor cache of derived values (diffrast _cache.py:16-82).

An entry is keyed on the tensor object's identity and remembers a weak reference and a stamp
(version counter, data pointer, shape). It is reused only while both match, so a tensor edited
in place, or a new tensor with the same contents, is computed again; the entry goes away with
the tensor. Writes that bypass the version counter (``tensor.data``, memory shared with NumPy)
are not noticed.
"""

from __future__ import annotations

import threading
import weakref
from collections import OrderedDict
from collections.abc import Callable
from typing import Generic, TypeVar

from torch import Tensor

T = TypeVar("T")


def stamp(tensor: Tensor) -> tuple | None:
    """What changes when ``tensor`` is modified or re-allocated; ``None`` for inference tensors."""
    if tensor.is_inference():
        return None
    return tensor._version, tensor.data_ptr(), tensor.shape


class TensorCache(Generic[T]):
    """``compute(tensor)`` remembered per tensor object, at most ``max_entries`` of them (LRU)."""

    def __init__(self, compute: Callable[[Tensor], T], max_entries: int = 64) -> None:
        self._compute = compute
        self._max_entries = max_entries
        self._entries: OrderedDict[int, tuple[weakref.ref, tuple, T]] = OrderedDict()
        # Re-entrant: a weak-reference callback may run while this thread holds the lock.
        self._lock = threading.RLock()

    def __len__(self) -> int:
        return len(self._entries)

    def get(self, tensor: Tensor) -> T:
        current = stamp(tensor)
        if current is None:
            return self._compute(tensor)
        key = id(tensor)
        entry = self._entries.get(key)
        if entry is not None and entry[0]() is tensor and entry[1] == current:
            return entry[2]
        value = self._compute(tensor)
        ref = weakref.ref(tensor, lambda r: self._discard(key, r))
        with self._lock:
            self._entries.pop(key, None)
            self._entries[key] = (ref, current, value)
            while len(self._entries) > self._max_entries:
                self._entries.popitem(last=False)
        return value

    def clear(self) -> None:
        with self._lock:
            self._entries.clear()

    def _discard(self, key: int, ref: weakref.ref) -> None:
        with self._lock:
            entry = self._entries.get(key)
            if entry is not None and entry[0] is ref:
                del self._entries[key]
