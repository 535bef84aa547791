"""Per-tensor memo of values derived from a tensor's contents (index ranges, range tables, edge
adjacency), with the caching behaviour diffrast documents for its ``TensorCache``
(diffrast ``_cache.py:30-82``): a value is reused only for the same tensor object while its
contents are unchanged, and is forgotten when that tensor is freed.

"Unchanged" is judged by a :class:`Signature`: the autograd version counter (bumped by every
in-place op, also through a view), the data address and the shape and strides. A tensor given
new storage, or edited in place, is therefore computed again. Writes that bypass the version
counter (through ``tensor.data`` or memory shared with NumPy) cannot be seen. Inference tensors
have no version counter and are never cached.

The memo is bounded: once ``max_entries`` tensors are remembered, the least recently used entry
is dropped (a hit counts as a use).
"""

from __future__ import annotations

import threading
import weakref
from collections.abc import Callable
from typing import Generic, NamedTuple, TypeVar

from torch import Tensor

T = TypeVar("T")


class Signature(NamedTuple):
    """What identifies the contents of a tensor object between two lookups."""

    version: int
    address: int
    shape: tuple
    strides: tuple


def signature(tensor: Tensor) -> Signature | None:
    """The :class:`Signature` of ``tensor``, or ``None`` when it has no version counter."""
    if tensor.is_inference():
        return None
    return Signature(tensor._version, tensor.data_ptr(), tuple(tensor.shape), tensor.stride())


class _Memo:
    """One remembered value: the tensor it belongs to (weakly) and the signature it had."""

    __slots__ = ("owner", "sig", "value")

    def __init__(self, owner: weakref.ref, sig: Signature, value) -> None:
        self.owner = owner
        self.sig = sig
        self.value = value

    def valid_for(self, tensor: Tensor, sig: Signature) -> bool:
        return self.owner() is tensor and self.sig == sig


class TensorCache(Generic[T]):
    """``compute(tensor)``, remembered for up to ``max_entries`` live tensor objects.

    ``compute``'s result must not hold a reference to the tensor, or the tensor is never freed.
    Lookups from several threads are safe; two threads that miss on the same tensor at once may
    both compute it.
    """

    def __init__(self, compute: Callable[[Tensor], T], max_entries: int = 64) -> None:
        if max_entries < 1:
            raise ValueError(f"max_entries must be at least 1, got {max_entries}.")
        self._compute = compute
        self._limit = max_entries
        # id(tensor) -> _Memo, least recently used first (dicts keep insertion order).
        self._memos: dict[int, _Memo] = {}
        # A weak-reference callback can run in the middle of a locked section of the same thread
        # (the garbage collector frees a tensor there), hence re-entrant.
        self._mutex = threading.RLock()

    def __len__(self) -> int:
        return len(self._memos)

    def get(self, tensor: Tensor) -> T:
        sig = signature(tensor)
        if sig is None:
            return self._compute(tensor)
        slot = id(tensor)
        with self._mutex:
            memo = self._memos.pop(slot, None)
            if memo is not None and memo.valid_for(tensor, sig):
                self._memos[slot] = memo  # now the most recently used
                return memo.value
        value = self._compute(tensor)
        owner = weakref.ref(tensor, self._forget_callback(slot))
        with self._mutex:
            self._memos.pop(slot, None)
            self._memos[slot] = _Memo(owner, sig, value)
            excess = len(self._memos) - self._limit
            for stale in list(self._memos)[:max(0, excess)]:
                del self._memos[stale]
        return value

    def clear(self) -> None:
        with self._mutex:
            self._memos.clear()

    def _forget_callback(self, slot: int) -> Callable[[weakref.ref], None]:
        # The callback holds the cache weakly, so a cache that goes away is not kept alive by the
        # tensors it once saw.
        cache = weakref.ref(self)

        def forget(dead: weakref.ref) -> None:
            owner = cache()
            if owner is None:
                return
            with owner._mutex:
                memo = owner._memos.get(slot)
                # The slot may already hold a newer tensor that got the same id.
                if memo is not None and memo.owner is dead:
                    del owner._memos[slot]

        return forget
