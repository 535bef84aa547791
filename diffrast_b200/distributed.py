"""Data parallelism over views: one process per GPU, views sharded, shared gradients summed.

Views are independent through the whole render path; the only coupling is the sum of gradients
of tensors shared by all views (the texture, a shared vertex buffer). A job of B views on N ranks
gives rank r the contiguous views ``view_shard(B, r, N)``; after the backward pass the gradients
of the shared tensors are summed with one all-reduce each (NCCL on GPUs, gloo on CPUs), issued in
buckets so that large textures pipeline over NVLink.
"""

from __future__ import annotations

import os

import torch
import torch.distributed as dist
from torch import Tensor


def init_process_group(device: torch.device, timeout_s: float = 300.0) -> None:
    """Join the job's process group (NCCL, rank and size from the environment) for view
    parallelism on ``device``.

    The NCCL collectives get a high-priority stream: the gradient all-reduces issued during the
    backward pass then take SMs as the running backward kernels' blocks finish, instead of waiting
    behind every block those kernels still have queued, so the transfer overlaps them.
    """
    from datetime import timedelta

    options = dist.ProcessGroupNCCL.Options(is_high_priority_stream=True)
    dist.init_process_group("nccl", timeout=timedelta(seconds=timeout_s), device_id=device,
                            pg_options=options)


def view_shard(num_views: int, rank: int, world_size: int) -> slice:
    """Views of ``rank``: contiguous, sizes differing by at most one, covering all ``num_views``."""
    if world_size < 1 or not 0 <= rank < world_size:
        raise ValueError(f"rank {rank} is not in a world of size {world_size}.")
    base, extra = divmod(num_views, world_size)
    start = rank * base + min(rank, extra)
    return slice(start, start + base + (1 if rank < extra else 0))


def sum_gradients(tensors: list[Tensor], group=None, bucket_bytes: int = 64 << 20) -> None:
    """All-reduce (sum) the ``.grad`` of every tensor in place, across ``group``.

    Gradients are reduced in chunks of at most ``bucket_bytes`` so that a 200 MB texture gradient
    is sent as several collectives that overlap each other's transfers. Tensors without a
    gradient take part with zeros, so every rank issues the same collectives in the same order.
    """
    if not dist.is_available() or not dist.is_initialized():
        return
    for t in tensors:
        if t.grad is None:
            t.grad = torch.zeros_like(t)
        flat = t.grad.view(-1)
        step = max(1, bucket_bytes // flat.element_size())
        for start in range(0, flat.numel(), step):
            dist.all_reduce(flat[start : start + step], group=group)


# Ranks from which OverlappedGradientSum splits the texture lookups' fused backward pass: the
# split costs a compact coordinate-gradient hand-over (on config 5, 1.96 + 0.86 ms against 2.63 ms
# fused on 2 GPUs) and hides the texture gradient's all-reduce behind the position part (exposed
# 0.47 -> 0.06 ms): 11.27 -> 11.01 ms per step on 2 GPUs, 6.20 -> 5.91 ms on 4.
DEFER_RANKS = 2


class OverlappedGradientSum:
    """Sums the gradients of shared tensors across ranks while the backward pass runs.

    A post-accumulate-grad hook on each tensor issues its bucketed all-reduces asynchronously as
    soon as the tensor's gradient is complete (the texture's, say, before the interpolation and
    rasterization backward passes run), so the transfers overlap the remaining kernels. Call
    :meth:`wait` after ``backward()`` and before reading the gradients; it also reduces, with
    zeros, the tensors that received no gradient, so that every rank issues the same
    collectives. Every rank must run the same graph (the hooks then fire in the same order).
    Without an initialised process group it does nothing. ``split_lookups`` (for a texture among
    ``tensors``) lets the lookups' backward passes complete the texture gradient first.
    """

    def __init__(self, tensors: list[Tensor], group=None, bucket_bytes: int = 64 << 20,
                 split_lookups: bool = True) -> None:
        self.tensors = list(tensors)
        self.group = group
        self.bucket_bytes = bucket_bytes
        self._pending: list = []
        self._done: set[int] = set()
        self._hooks = [t.register_post_accumulate_grad_hook(self._reduce) for t in self.tensors]
        if self._active() and split_lookups:
            # From DEFER_RANKS ranks on, texture lookups complete the texture gradient before
            # their position gradient work (which then runs in the interpolation's backward pass),
            # so that the texture's all-reduce overlaps it (see
            # diffrast_b200._functions.DEFER_CHAINED_BACKWARD); DIFFRAST_B200_DEFER_CHAINED=0/1
            # overrides.
            from diffrast_b200 import _functions

            forced = os.environ.get("DIFFRAST_B200_DEFER_CHAINED")
            ranks = dist.get_world_size(group)
            _functions.DEFER_CHAINED_BACKWARD = (forced != "0") if forced else ranks >= DEFER_RANKS

    def _active(self) -> bool:
        return dist.is_available() and dist.is_initialized()

    def _reduce(self, t: Tensor) -> None:
        if not self._active() or id(t) in self._done:
            return
        self._done.add(id(t))
        flat = t.grad.view(-1)
        step = max(1, self.bucket_bytes // flat.element_size())
        for start in range(0, flat.numel(), step):
            self._pending.append(
                dist.all_reduce(flat[start : start + step], group=self.group, async_op=True)
            )

    def wait(self) -> None:
        """Completes the reductions of this backward pass (the current stream waits for them)."""
        if not self._active():
            return
        for t in self.tensors:
            if id(t) not in self._done:
                if t.grad is None:
                    t.grad = torch.zeros_like(t)
                self._reduce(t)
        for work in self._pending:
            work.wait()
        self._pending.clear()
        self._done.clear()

    def remove(self) -> None:
        """Detaches the hooks."""
        for h in self._hooks:
            h.remove()
        self._hooks.clear()


class NextStepGradientSum:
    """Sums a tensor's gradient across ranks while the next step's forward pass runs, up to the
    tensor's first use in that step.

    The texture of a render-and-fit step is first read by the texture lookup, after the transform,
    the rasterization and the interpolation, none of which needs it. Its gradient sum can
    therefore run during those passes instead of after the backward pass, where little work is
    left to hide it behind: :meth:`hold` at the end of a step copies the local gradient into a
    reduction buffer, :meth:`start` at the start of the next step issues its all-reduces, and
    :meth:`wait`, before the tensor's first use (after which an optimizer would apply
    :attr:`buffer`), completes them. This is the order of synchronous data parallelism, with the
    sum moved from the end of one step to the start of the next; after the last step, :meth:`start`
    and :meth:`wait` complete the last sum. Every rank must make the same calls. Without an
    initialised process group it only copies.
    """

    def __init__(self, tensor: Tensor, group=None, bucket_bytes: int = 64 << 20) -> None:
        self.tensor = tensor
        self.group = group
        self.bucket_bytes = bucket_bytes
        self.buffer: Tensor | None = None
        self._held = False
        self._work: list = []

    def _active(self) -> bool:
        return dist.is_available() and dist.is_initialized()

    def hold(self) -> None:
        """Takes this step's local gradient (zeros when there is none) for the next sum."""
        if self.buffer is None:
            self.buffer = torch.zeros_like(self.tensor)
        if self.tensor.grad is None:
            self.buffer.zero_()
        else:
            self.buffer.copy_(self.tensor.grad)
        self._held = True

    def start(self) -> None:
        """Issues the all-reduces of the held gradient, asynchronously (nothing when none is held)."""
        if not self._held:
            return
        self._held = False
        if not self._active():
            return
        flat = self.buffer.view(-1)
        step = max(1, self.bucket_bytes // flat.element_size())
        for first in range(0, flat.numel(), step):
            self._work.append(
                dist.all_reduce(flat[first : first + step], group=self.group, async_op=True)
            )

    def wait(self) -> None:
        """Completes the sum (the current stream waits for it): :attr:`buffer` then holds the
        previous step's gradient summed over the ranks."""
        for work in self._work:
            work.wait()
        self._work.clear()
