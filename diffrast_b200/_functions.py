"""Autograd functions over the CUDA kernels. Inputs arrive validated (see ``ops.py``).

Each backward runs hand-written kernels with no second-order terms, so a backward pass asked to
build a graph (``create_graph=True``) raises, like the reference's first-order guard
(diffrast backends/_autograd.py:11-35).
"""

from __future__ import annotations

import functools
import weakref
from typing import NamedTuple

import torch
from torch import Tensor

from diffrast_b200 import _kernels as K


def first_order(op: str):
    def decorate(backward):
        @functools.wraps(backward)
        def guarded(ctx, *grads):
            if torch.is_grad_enabled():
                raise RuntimeError(
                    f"{op} in diffrast_b200 has no second-order gradients, but its backward pass "
                    "was run with create_graph=True."
                )
            return backward(ctx, *grads)

        return guarded

    return decorate


def _saveable(t: Tensor | None) -> Tensor | None:
    # A tensor made in inference mode cannot be saved for backward, but a copy of it can.
    return t.clone() if t is not None and t.is_inference() else t


def _take(src: Tensor | None, spec: tuple[int, int] | None) -> Tensor | None:
    """``src`` itself, or its channels ``spec = (first, count)`` when the lookup input was passed
    as the wider tensor it is a slice of."""
    return src if src is None or spec is None else src[..., spec[0]:spec[0] + spec[1]]


def _slice_gradient(src: Tensor, spec: tuple[int, int] | None, want: bool):
    """(gradient of ``src``, its first lookup channel) for an input passed with a channel ``spec``:
    the kernel writes whole pixel records, zero outside the slice. (None, -1) otherwise."""
    if not want or spec is None:
        return None, -1
    return torch.empty(src.shape, dtype=src.dtype, device=src.device), spec[0]


class CoordinatePort:
    """Hand-over of compact coordinate gradients from texture lookups to the interpolation whose
    output channels they read.

    ``interpolate`` returns, next to ``out`` and ``out_da``, a zero-size ``sink`` tensor of its
    autograd node, and attaches this port to both outputs. A lookup given channel slices of them
    (``out[..., 0:2]``, ``out_da[..., 0:4]``) depends on ``sink`` instead of the outputs; its
    backward pass leaves its compact uv / uv_da gradients in ``pending`` and returns an empty
    gradient for ``sink``, and the interpolation's backward pass reads them from there. So no
    zero-padded gradient records of the whole outputs are written or read. Entries are tagged
    with the autograd graph task that made them: a backward pass only ever uses its own.

    The port also describes the interpolation (``geometry``, set by its forward pass), so that a
    2D lookup can run the interpolation's backward pass for its coordinates inside its own
    (``dr_texture_bwd_interp``) and hand over gradients of rast and rast_db instead
    (:class:`Chained`).
    """

    def __init__(self, sink: Tensor | None, pending: dict, diff_channels: tuple = ()) -> None:
        self.sink = sink
        self.pending = pending
        self.diff_channels = diff_channels
        self.geometry: InterpGeometry | None = None


class InterpGeometry:
    """What produced an interpolation's outputs, as the fused texture backward pass reads it:
    ``attr`` ``[batch or 1, vertices, channels]`` (contiguous), ``rast``, ``tri``, and whether
    attr needs a gradient (the fused pass computes none). The tensors are the interpolation's
    saved tensors; its backward pass releases them here (a later backward pass through a retained
    graph then hands over compact coordinate gradients instead), so that the outputs, which keep
    the port, do not keep them alive after the graph has freed its own copies."""

    def __init__(self, attr: Tensor, rast: Tensor, tri: Tensor, attr_needs_grad: bool) -> None:
        self._tensors: tuple | None = (attr, rast, tri)
        self.attr_needs_grad = attr_needs_grad

    def tensors(self):
        """``(attr, rast, tri)``, or None once released."""
        return self._tensors

    def release(self) -> None:
        self._tensors = None


class Chained(NamedTuple):
    """A lookup's coordinate gradients already chained through the interpolation: gradients of
    rast and rast_db (``grad_db`` None when uv_da got none)."""

    grad_rast: Tensor
    grad_db: Tensor | None


class RasterChain(NamedTuple):
    """The rasterization part of a fused texture backward pass: the clip positions and keys the
    rasterizer used, whether rast_db's gradient reaches the positions, and the position gradient
    buffer to accumulate into."""

    pos: Tensor
    keys: Tensor
    grad_db: bool
    grad_pos: Tensor


class ChainArgs(NamedTuple):
    """Arguments of the fused texture backward pass: the interpolation's tensors and the
    attribute channels of uv (cu, cv) and of uv_da's two derivative pairs (du, dv); with
    ``raster``, the rasterizer's backward pass runs in it as well."""

    attr: Tensor
    rast: Tensor
    tri: Tensor
    cu: int
    cv: int
    du: int
    dv: int
    raster: RasterChain | None = None


# Whether 2D lookups of interpolated coordinates run the interpolation's backward pass for them
# inside their own, and whether they run the rasterizer's backward pass there too when the
# interpolation read rasterize's own rast (tests switch them off to compare against the
# separate passes).
FUSE_INTERPOLATION_BACKWARD = True
FUSE_RASTERIZE_BACKWARD = True
# Whether a lookup that would run the rasterizer's backward pass in its own splits it instead:
# texel and compact coordinate gradients in its own backward pass, the chained position part
# (dr_texture_chain_bwd) in the interpolation's, which autograd runs after the texture's gradient
# is complete. The texture gradient is then final, and can be reduced across GPUs while the
# position part runs; one fused pass is faster where nothing waits for the texture gradient.
# diffrast_b200.distributed.OverlappedGradientSum turns it on when it sums across ranks.
DEFER_CHAINED_BACKWARD = False


class Deferred(NamedTuple):
    """A lookup's chained position part, left for the interpolation's backward pass to run: its
    compact coordinate gradients and the chain (``dr_texture_chain_bwd``)."""

    g_uv: Tensor
    g_da: Tensor | None
    want_da: bool
    chain: ChainArgs


def _run_deferred(d: Deferred) -> Chained:
    K.texture_chain_bwd(d.g_uv, d.g_da, d.want_da, d.chain)
    return Chained(None, None)


class Route:
    """How a lookup's coordinate gradients leave it: through ``pending`` of a
    :class:`CoordinatePort`, for uv and uv_da as requested at the forward pass."""

    def __init__(self, pending: dict, want_uv: bool, want_da: bool,
                 port: CoordinatePort | None = None, pos_port: PositionPort | None = None) -> None:
        self.pending = pending
        self.want_uv = want_uv
        self.want_da = want_da
        self.port = port
        # The rasterization that made the interpolation's rast, when the lookup depends on its
        # sink (so that the rasterizer's backward pass runs and collects the position gradient).
        self.pos_port = pos_port

    def deliver(self, key, uv_first, g_uv, da_first, g_da) -> None:
        self.pending[(torch._C._current_graph_task_id(), key)] = (uv_first, g_uv, da_first, g_da)

    def deliver_chained(self, key, grad_rast, grad_db) -> None:
        self.pending[(torch._C._current_graph_task_id(), key)] = Chained(grad_rast, grad_db)

    def deliver_deferred(self, key, deferred: Deferred) -> None:
        self.pending[(torch._C._current_graph_task_id(), key)] = deferred

    def chain(self, uv_spec, da_spec, mode: int, boundary: int, want_da: bool) -> ChainArgs | None:
        """The fused backward pass's arguments when it applies: a 2D lookup of two consecutive
        interpolated channels (and of two whole derivative pairs), an interpolation whose
        attributes need no gradient and whose tensors are alive, and no other lookup of this
        backward pass fused with the same interpolation. None otherwise."""
        port = self.port
        if (not FUSE_INTERPOLATION_BACKWARD or port is None or port.geometry is None
                or boundary == 3 or mode < 1 or uv_spec is None or uv_spec[1] != 2
                or port.geometry.attr_needs_grad):
            return None
        if want_da and (da_spec is None or da_spec[1] != 4 or da_spec[0] % 2
                        or da_spec[0] // 2 + 2 > len(port.diff_channels)):
            return None
        task = torch._C._current_graph_task_id()
        if any(k[0] == task and isinstance(v, (Chained, Deferred)) for k, v in self.pending.items()):
            return None
        got = port.geometry.tensors()
        if got is None:
            return None
        attr, rast, tri = got
        du = dv = 0
        if want_da:
            du = port.diff_channels[da_spec[0] // 2]
            dv = port.diff_channels[da_spec[0] // 2 + 1]
        raster = self._raster_chain(rast, tri, task)
        if DEFER_CHAINED_BACKWARD and raster is None:
            return None  # deferred: the interpolation's backward pass takes compact parts
        return ChainArgs(attr, rast, tri, uv_spec[0], uv_spec[0] + 1, du, dv, raster)

    def _raster_chain(self, rast, tri, task) -> RasterChain | None:
        """The rasterization part when it applies: the interpolation read the very rast of a
        rasterize call over the same tri, whose sink this lookup depends on. The position
        gradient buffer is the one antialias already left for that rasterization in this backward
        pass, or a new zeroed one left there."""
        pp = self.pos_port
        if not FUSE_RASTERIZE_BACKWARD or pp is None or pp.raster is None:
            return None
        r = pp.raster.tensors()
        if r is None or getattr(rast, "_dr_pos_port", None) is not pp:
            return None
        pos, r_tri, keys, grad_db = r
        if r_tri is not tri:
            return None
        grad_pos = next((v for k, v in pp.pending.items() if k[0] == task), None)
        if grad_pos is None:
            grad_pos = K.zeros(pos.shape, pos.device)
            pp.pending[(task, id(self))] = grad_pos
        return RasterChain(pos, keys, grad_db, grad_pos)


def _take_pending(pending: dict) -> list:
    """The hand-overs delivered to ``pending`` in the running backward pass; clears ``pending``
    (entries of other, finished passes are stale, and dropping them frees their gradients). Two
    backward passes through the same graph must therefore not run at the same time (in two
    threads); one after the other, with ``retain_graph=True``, they are independent."""
    task = torch._C._current_graph_task_id()
    mine = [v for k, v in pending.items() if k[0] == task]
    pending.clear()
    return mine


class PositionPort:
    """Hand-over of antialias's position gradient to the rasterization that made its ``rast``.

    Both ops differentiate the same clip positions; without the hand-over, each fills a gradient
    buffer of the positions' size with zeros, scatters into it, and autograd adds the two. With
    it, ``rasterize`` returns a zero-size ``sink`` next to rast, rast_db and the keys, and this
    port is attached to rast; an antialias pass given that rast and the same ``pos`` tensor
    depends on ``sink`` instead of ``pos``, leaves its position gradient in ``pending``, and the
    rasterizer's backward pass accumulates its own scatter into that buffer.

    It also describes the rasterization (``raster``, set by its forward pass) for a texture
    lookup of coordinates interpolated from this rast, which can run the rasterizer's backward
    pass inside its own (:meth:`Route.chain`).
    """

    def __init__(self, sink: Tensor | None, pending: dict, pos: Tensor) -> None:
        self.sink = sink
        self.pending = pending
        self.pos = weakref.ref(pos)
        self.raster: RasterGeometry | None = None


class RasterGeometry:
    """The rasterizer's clip positions (as its kernels read them), tri, keys and whether rast_db
    is differentiable; its backward pass releases them here, like :class:`InterpGeometry`."""

    def __init__(self, pos: Tensor, tri: Tensor, keys: Tensor, grad_db: bool) -> None:
        self._tensors: tuple | None = (pos, tri, keys, grad_db)

    def tensors(self):
        """``(pos, tri, keys, grad_db)``, or None once released."""
        return self._tensors

    def release(self) -> None:
        self._tensors = None


def _collect(pending: dict, channels: int, da_channels: int, grad_out, grad_out_da):
    """The coordinate gradients delivered in this backward pass (consumed), as at most one compact
    part per output plus whole images for anything that does not fit that form, and the
    hand-overs already chained through the interpolation (:class:`Chained`)."""
    mine = [_run_deferred(v) if isinstance(v, Deferred) else v for v in _take_pending(pending)]
    chained = [v for v in mine if isinstance(v, Chained)]
    parts: dict[str, tuple[int, Tensor]] = {}
    for uv_first, g_uv, da_first, g_da in (v for v in mine if not isinstance(v, Chained)):
        for name, first, g in (("out", uv_first, g_uv), ("da", da_first, g_da)):
            if g is None:
                continue
            held = parts.get(name)
            if held is None:
                parts[name] = (first, g)
            elif held[0] == first and held[1].shape == g.shape:
                parts[name] = (first, held[1] + g)
            else:  # different channel ranges: fold into the whole image
                width = channels if name == "out" else da_channels
                full = grad_out if name == "out" else grad_out_da
                if full is None:
                    full = torch.zeros((*g.shape[:3], width), device=g.device)
                else:
                    full = full.clone()
                full[..., first:first + g.shape[-1]] += g
                if name == "out":
                    grad_out = full
                else:
                    grad_out_da = full
    return parts.get("out"), parts.get("da"), grad_out, grad_out_da, chained


class Rasterize(torch.autograd.Function):
    """Visibility, then rast / rast_db; gradients reach pos through the barycentric resolve.
    Returns ``(rast, rast_db, keys, sink)``; ``sink`` receives antialias's position gradient
    (:class:`PositionPort`)."""

    @staticmethod
    def forward(ctx, pos: Tensor, tri: Tensor, height: int, width: int, grad_db: bool,
                prev_keys: Tensor | None, ranges: K.RangeTable | None, port: PositionPort):
        keys = K.raster_keys(pos, tri, height, width, prev_keys, ranges)
        rast, rast_db = K.resolve_fwd(pos, tri, keys)
        # Unused outputs (keys always, rast_db often) get no zero-filled gradient.
        ctx.set_materialize_grads(False)
        saved = (_saveable(pos), _saveable(tri), keys)
        ctx.save_for_backward(*saved)
        ctx.grad_db = grad_db
        ctx.pending = port.pending
        ctx.geometry = None
        if ranges is None:
            ctx.geometry = port.raster = RasterGeometry(saved[0], saved[1], keys, grad_db)
        ctx.mark_non_differentiable(keys)
        if not grad_db:
            ctx.mark_non_differentiable(rast_db)
        return rast, rast_db, keys, pos.new_empty(0)

    @staticmethod
    @first_order("rasterize")
    def backward(ctx, grad_rast, grad_db, _grad_keys, grad_sink):
        pos, tri, keys = ctx.saved_tensors
        if ctx.geometry is not None:
            ctx.geometry.release()
        start = None
        if grad_sink is not None:
            for g in _take_pending(ctx.pending):
                start = g if start is None else start + g
        use_db = ctx.grad_db and grad_db is not None
        if grad_rast is None and not use_db and start is not None:
            grad_pos = start
        else:
            if grad_rast is None:
                grad_rast = torch.zeros((*keys.shape, 4), dtype=pos.dtype, device=pos.device)
            grad_pos = K.resolve_bwd(pos, tri, keys, K.aligned(grad_rast),
                                     K.aligned(grad_db) if use_db else None, start=start)
        return grad_pos, None, None, None, None, None, None, None


class Interpolate(torch.autograd.Function):
    """Returns ``(out, out_da, sink)``: ``sink`` is the zero-size tensor through which lookups
    that read channel slices of the outputs hand their gradients back (:class:`CoordinatePort`)."""

    @staticmethod
    def forward(ctx, attr: Tensor, rast: Tensor, rast_db: Tensor | None, tri: Tensor,
                diff: Tensor | None, port: CoordinatePort):
        attr3 = (attr if attr.ndim == 3 else attr[None]).contiguous()
        channels = attr3.shape[2]
        # Rows padded to 16 bytes for the forward kernel's vector loads.
        attr_rows, _ = K.padded_rows(attr3)
        out, out_da = K.interpolate_fwd(attr_rows, rast, rast_db, tri, diff, channels)
        ctx.set_materialize_grads(False)
        saved = tuple(_saveable(t) for t in (attr3, rast, rast_db, tri, diff))
        ctx.save_for_backward(*saved)
        ctx.attr_shape = attr.shape
        ctx.channels = channels
        ctx.has_da = diff is not None
        ctx.rast_db_given = rast_db is not None
        ctx.pending = port.pending
        ctx.geometry = port.geometry = InterpGeometry(saved[0], saved[1], saved[3],
                                                      ctx.needs_input_grad[0])
        if diff is None:
            ctx.mark_non_differentiable(out_da)
        return out, out_da, rast.new_empty(0)

    @staticmethod
    @first_order("interpolate")
    def backward(ctx, grad_out, grad_out_da, grad_sink):
        attr3, rast, rast_db, tri, diff = ctx.saved_tensors
        ctx.geometry.release()
        part = part_da = None
        chained: list[Chained] = []
        if grad_sink is not None:
            num_da = 0 if diff is None else 2 * diff.shape[0]
            part, part_da, grad_out, grad_out_da, chained = _collect(
                ctx.pending, ctx.channels, num_da, grad_out, grad_out_da)
        need_attr = ctx.needs_input_grad[0]
        c_rast = c_db = None
        for c in chained:  # (None, None): the lookup went on through the rasterizer too
            if c.grad_rast is not None:
                c_rast = c.grad_rast if c_rast is None else c_rast + c.grad_rast
            if c.grad_db is not None:
                c_db = c.grad_db if c_db is None else c_db + c.grad_db
        if chained and part is None and part_da is None and grad_out is None \
                and grad_out_da is None and not need_attr:
            # Everything was chained inside the lookups' backward passes.
            return None, c_rast, c_db if ctx.rast_db_given else None, None, None, None
        use_da = ctx.has_da and (grad_out_da is not None or part_da is not None)
        if not use_da:
            grad_out_da = part_da = None
        grad_attr, grad_rast, grad_db = K.interpolate_bwd(
            attr3, rast, rast_db, tri, diff if use_da else None,
            None if grad_out is None else grad_out.contiguous(),
            grad_out_da.contiguous() if grad_out_da is not None else None, need_attr,
            part=None if part is None else part[1].contiguous(),
            part_first=0 if part is None else part[0],
            part_da=None if part_da is None else part_da[1].contiguous(),
            da_first=0 if part_da is None else part_da[0],
        )
        if c_rast is not None:
            grad_rast = c_rast if grad_rast is None else grad_rast.add_(c_rast)
        if c_db is not None:
            grad_db = c_db if grad_db is None else grad_db.add_(c_db)
        if not ctx.rast_db_given:
            grad_db = None
        if grad_attr is not None:
            grad_attr = grad_attr.view(ctx.attr_shape)
        return grad_attr, grad_rast, grad_db, None, None, None


class MipChain(torch.autograd.Function):
    """Levels 1.. of a texture by repeated area-weighted halving; backward is the adjoint chain."""

    @staticmethod
    def forward(ctx, tex: Tensor, count: int):
        levels = K.mip_build(tex, count)
        ctx.shapes = [tex.shape, *(lv.shape for lv in levels)]
        ctx.device = tex.device
        return tuple(levels)

    @staticmethod
    @first_order("texture_construct_mip")
    def backward(ctx, *grads):
        shapes = ctx.shapes
        # Gradient of the coarsest level first, pushed down one step at a time.
        carry = None
        for index in range(len(shapes) - 1, 0, -1):
            g = grads[index - 1]
            g = torch.zeros(shapes[index], device=ctx.device) if g is None else g.contiguous().clone()
            if carry is not None:
                g += carry
            fine = torch.zeros(shapes[index - 1], device=ctx.device)
            K.mip_down_bwd(g, fine)
            carry = fine
        return carry, None


class Texture(torch.autograd.Function):
    """Lookup in a list of levels (base texture first); gradients to every level and to uv,
    uv_da and the level-of-detail bias as the filter mode allows.

    uv and uv_da may be passed as the wider tensors they are channel slices of (``uv_spec`` /
    ``da_spec`` = (first channel, count)), such as interpolate's outputs. With a ``route`` (the
    outputs of :func:`diffrast_b200.interpolate`), they arrive detached and their compact
    gradients go back through the interpolation's :class:`CoordinatePort` (``sink`` is its
    zero-size tensor); otherwise the gradients are written straight into gradients of the wider
    tensors instead of being copied there by the slices' own backward."""

    @staticmethod
    def forward(ctx, uv_src, da_src, bias, mode: int, boundary: int, uv_spec, da_spec, route,
                sink, pos_sink, *levels):
        levels = [lv.contiguous() for lv in levels]
        out = K.texture_fwd(list(levels), _take(uv_src, uv_spec), _take(da_src, da_spec), bias,
                            mode, boundary)
        ctx.save_for_backward(*(_saveable(t) for t in (uv_src, da_src, bias, *levels)))
        ctx.settings = (mode, boundary, da_src is not None, bias is not None, len(levels))
        ctx.specs = (uv_spec, da_spec)
        ctx.route = route
        return out

    @staticmethod
    @first_order("texture")
    def backward(ctx, grad_out):
        mode, boundary, has_da, has_bias, count = ctx.settings
        uv_spec, da_spec = ctx.specs
        route = ctx.route
        saved = ctx.saved_tensors
        uv_src, da_src, bias, levels = saved[0], saved[1], saved[2], list(saved[3:])
        need = ctx.needs_input_grad
        want_uv = (route.want_uv if route is not None else need[0]) and mode > 0
        want_da = (route.want_da if route is not None else need[1]) and has_da and mode == 3
        want_bias = need[2] and has_bias and mode == 3
        g_uv_src = g_da_src = None
        uv_first = da_first = -1
        if route is None:
            g_uv_src, uv_first = _slice_gradient(uv_src, uv_spec, want_uv)
            g_da_src, da_first = _slice_gradient(da_src, da_spec, want_da)
        chain = route.chain(uv_spec, da_spec, mode, boundary, want_da) if route is not None else None
        deferred = chain is not None and DEFER_CHAINED_BACKWARD
        if deferred:
            grads, g_uv, g_da, g_bias = K.texture_bwd(
                levels, _take(uv_src, uv_spec), _take(da_src, da_spec), bias, mode, boundary,
                grad_out.contiguous(), True, want_da, want_bias)
        elif chain is not None:
            grads, g_rast, g_db, g_bias = K.texture_bwd_chained(
                levels, _take(uv_src, uv_spec), _take(da_src, da_spec), bias, mode, boundary,
                grad_out.contiguous(), want_da, want_bias, chain)
        else:
            grads, g_uv, g_da, g_bias = K.texture_bwd(
                levels, _take(uv_src, uv_spec), _take(da_src, da_spec), bias, mode, boundary,
                grad_out.contiguous(), want_uv, want_da, want_bias, grad_uv=g_uv_src,
                grad_da=g_da_src, uv_first=uv_first, da_first=da_first)
        level_grads = [g if need[10 + i] else None for i, g in enumerate(grads)]
        if route is not None:
            if deferred:
                route.deliver_deferred(id(ctx), Deferred(g_uv, g_da, want_da, chain))
            elif chain is not None:
                route.deliver_chained(id(ctx), g_rast, g_db)
            else:
                route.deliver(id(ctx), uv_spec[0], g_uv,
                              None if da_spec is None else da_spec[0], g_da)
            sink = grad_out.new_empty(0) if need[8] else None
            pos_sink = grad_out.new_empty(0) if need[9] and chain is not None \
                and chain.raster is not None else None
            return (None, None, g_bias, None, None, None, None, None, sink, pos_sink,
                    *level_grads)
        g_uv = g_uv_src if uv_spec is not None else g_uv
        g_da = g_da_src if da_spec is not None else g_da
        return (g_uv, g_da, g_bias, None, None, None, None, None, None, None, *level_grads)


class TextureChain(torch.autograd.Function):
    """Mipmapped lookup with the mip chain of ``tex`` built inside the function.

    The levels never enter the autograd graph: the backward pass accumulates the gradients of all
    levels (in 4-channel buffers when the texture has 3 channels), pushes them down the chain with
    the adjoint kernel in place, and returns only the base level's gradient.
    """

    @staticmethod
    def forward(ctx, uv_src, da_src, bias, mode: int, boundary: int, count: int, tex: Tensor,
                uv_spec=None, da_spec=None, route=None, sink=None, pos_sink=None):
        tex = tex.contiguous()
        levels = [tex, *K.mip_build(tex, count)]
        out = K.texture_fwd(levels, _take(uv_src, uv_spec), _take(da_src, da_spec), bias, mode,
                            boundary)
        ctx.save_for_backward(*(_saveable(t) for t in (uv_src, da_src, bias, tex)))
        ctx.levels = levels[1:]
        ctx.settings = (mode, boundary)
        ctx.specs = (uv_spec, da_spec)
        ctx.route = route
        return out

    @staticmethod
    @first_order("texture")
    def backward(ctx, grad_out):
        mode, boundary = ctx.settings
        uv_spec, da_spec = ctx.specs
        route = ctx.route
        uv_src, da_src, bias, tex = ctx.saved_tensors
        levels = [tex, *ctx.levels]
        need = ctx.needs_input_grad
        want_uv = (route.want_uv if route is not None else need[0]) and mode > 0
        want_da = ((route.want_da if route is not None else need[1]) and da_src is not None
                   and mode == 3)
        want_bias = need[2] and bias is not None and mode == 3
        g_uv_src = g_da_src = None
        uv_first = da_first = -1
        if route is None:
            g_uv_src, uv_first = _slice_gradient(uv_src, uv_spec, want_uv)
            g_da_src, da_first = _slice_gradient(da_src, da_spec, want_da)
        chain = route.chain(uv_spec, da_spec, mode, boundary, want_da) if route is not None else None
        deferred = chain is not None and DEFER_CHAINED_BACKWARD
        if deferred:
            grads, g_uv, g_da, g_bias = K.texture_bwd(
                levels, _take(uv_src, uv_spec), _take(da_src, da_spec), bias, mode, boundary,
                grad_out.contiguous(), True, want_da, want_bias, keep_padded=True)
        elif chain is not None:
            grads, g_rast, g_db, g_bias = K.texture_bwd_chained(
                levels, _take(uv_src, uv_spec), _take(da_src, da_spec), bias, mode, boundary,
                grad_out.contiguous(), want_da, want_bias, chain, keep_padded=True)
        else:
            grads, g_uv, g_da, g_bias = K.texture_bwd(
                levels, _take(uv_src, uv_spec), _take(da_src, da_spec), bias, mode, boundary,
                grad_out.contiguous(), want_uv, want_da, want_bias, keep_padded=True,
                grad_uv=g_uv_src, grad_da=g_da_src, uv_first=uv_first, da_first=da_first)
        grad_tex = None
        if need[6]:
            padded = grads[0].shape[-1] != tex.shape[-1]
            if len(grads) > 1:
                # The whole adjoint chain at once; with padding, the base gradient is written
                # without the padding channel.
                out = torch.empty(tex.shape, dtype=torch.float32, device=tex.device) if padded else None
                K.mip_build_bwd(grads, out)
                if padded:
                    grads[0] = out
            grad_tex = grads[0]
            if grad_tex.shape[-1] != tex.shape[-1]:
                grad_tex = grad_tex[..., : tex.shape[-1]].contiguous()
        if route is not None:
            if deferred:
                route.deliver_deferred(id(ctx), Deferred(g_uv, g_da, want_da, chain))
            elif chain is not None:
                route.deliver_chained(id(ctx), g_rast, g_db)
            else:
                route.deliver(id(ctx), uv_spec[0], g_uv,
                              None if da_spec is None else da_spec[0], g_da)
            sink = grad_out.new_empty(0) if need[10] else None
            pos_sink = grad_out.new_empty(0) if need[11] and chain is not None \
                and chain.raster is not None else None
            return None, None, g_bias, None, None, None, grad_tex, None, None, None, sink, pos_sink
        g_uv = g_uv_src if uv_spec is not None else g_uv
        g_da = g_da_src if da_spec is not None else g_da
        return g_uv, g_da, g_bias, None, None, None, grad_tex, None, None, None, None, None


def _deliver(route, grad_pos):
    """Leave ``grad_pos`` for the rasterizer (``route`` is its port's ``pending``)."""
    route[(torch._C._current_graph_task_id(), id(grad_pos))] = grad_pos


class Antialias(torch.autograd.Function):
    """With a ``route`` (``pending`` of a :class:`PositionPort`; ``pos`` then arrives detached and
    ``sink`` is the port's), the position gradient goes to the rasterizer's backward pass."""

    @staticmethod
    def forward(ctx, color: Tensor, rast: Tensor, pos: Tensor, tri: Tensor, opposite: Tensor,
                boost: float, route=None, sink=None):
        pos3 = pos if pos.ndim == 3 else pos[None]
        # The pair records (about 25 bytes per pixel) spare the backward pass the edge tests.
        out, pairs = K.antialias_fwd(color, rast, pos3, tri, opposite,
                                     record_pairs=any(ctx.needs_input_grad[:3]) or route is not None)
        saved = (color, rast, pos3, tri, opposite, pairs)
        ctx.save_for_backward(*(_saveable(t) for t in saved))
        ctx.boost = boost
        ctx.pos_shape = pos.shape
        ctx.route = route
        return out

    @staticmethod
    @first_order("antialias")
    def backward(ctx, grad_out):
        color, rast, pos3, tri, opposite, pairs = ctx.saved_tensors
        grad_color, grad_pos = K.antialias_bwd(color, rast, pos3, tri, opposite,
                                               grad_out.contiguous(), ctx.boost, pairs)
        grad_pos = grad_pos.view(ctx.pos_shape)
        if ctx.route is not None:
            _deliver(ctx.route, grad_pos)
            return grad_color, None, None, None, None, None, None, grad_pos.new_empty(0)
        return grad_color, None, grad_pos, None, None, None, None, None


class AntialiasMSE(torch.autograd.Function):
    """Antialias with the squared-error loss ``scale * sum (out - target)^2`` fused into its
    passes; returns ``(out, loss)``. ``route`` / ``sink`` as for :class:`Antialias`."""

    @staticmethod
    def forward(ctx, color: Tensor, rast: Tensor, pos: Tensor, tri: Tensor, opposite: Tensor,
                target: Tensor, scale: float, boost: float, route=None, sink=None):
        pos3 = pos if pos.ndim == 3 else pos[None]
        out, residual, pairs, partial = K.antialias_mse_fwd(color, rast, pos3, tri, opposite, target)
        loss = partial.sum() * scale
        ctx.set_materialize_grads(False)
        saved = (color, rast, pos3, tri, opposite, pairs, residual)
        ctx.save_for_backward(*(_saveable(t) for t in saved))
        ctx.scale, ctx.boost, ctx.pos_shape = scale, boost, pos.shape
        ctx.route = route
        return out, loss

    @staticmethod
    @first_order("antialias_mse")
    def backward(ctx, grad_out, grad_loss):
        color, rast, pos3, tri, opposite, pairs, residual = ctx.saved_tensors
        if grad_loss is None:
            grad_loss = torch.zeros((), dtype=torch.float32, device=color.device)
        grad_color, grad_pos = K.antialias_mse_bwd(
            color, rast, pos3, tri, opposite, residual, grad_loss.detach().float().contiguous(),
            ctx.scale, None if grad_out is None else grad_out.contiguous(), ctx.boost, pairs)
        grad_pos = grad_pos.view(ctx.pos_shape)
        if ctx.route is not None:
            _deliver(ctx.route, grad_pos)
            return (grad_color, None, None, None, None, None, None, None, None,
                    grad_pos.new_empty(0))
        return grad_color, None, grad_pos, None, None, None, None, None, None, None


class Lambert(torch.autograd.Function):
    """Lambert shading of ``color`` by the unit normal and light; the light is a constant."""

    @staticmethod
    def forward(ctx, color: Tensor, normal: Tensor, light: Tensor, ambient: float):
        out = K.lambert_fwd(color, normal, light, ambient)
        ctx.save_for_backward(*(_saveable(t) for t in (color, normal, light)))
        ctx.ambient = ambient
        return out

    @staticmethod
    @first_order("lambert")
    def backward(ctx, grad_out):
        color, normal, light = ctx.saved_tensors
        need = ctx.needs_input_grad
        grad_color, grad_normal = K.lambert_bwd(color, normal, light, ctx.ambient,
                                                grad_out.contiguous(), need[0], need[1])
        return grad_color, grad_normal, None, None


class ToClip(torch.autograd.Function):
    """World-to-clip transform of shared positions by per-view matrices."""

    @staticmethod
    def forward(ctx, positions: Tensor, matrix: Tensor):
        clip = K.to_clip_fwd(positions, matrix)
        ctx.save_for_backward(_saveable(positions), _saveable(matrix))
        return clip

    @staticmethod
    @first_order("to_clip")
    def backward(ctx, grad_clip):
        positions, matrix = ctx.saved_tensors
        grad_p, grad_m = K.to_clip_bwd(K.aligned(grad_clip), positions, matrix,
                                       ctx.needs_input_grad[0], ctx.needs_input_grad[1])
        return grad_p, grad_m
