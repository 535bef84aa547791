"""Public differentiable rasterization ops of diffrast_b200.

Signatures, argument meaning, validation and error messages follow diffrast's public API
(``src/diffrast/ops.py:29-638``), so code switches by changing its import. Every op runs on the
hand-written sm_100a kernels of ``libdiffrast_b200.so`` through autograd functions; there is no
other backend and no CPU fallback: tensors on the CPU pass validation and then raise
``RuntimeError``.
"""

from __future__ import annotations

import operator
from collections.abc import Sequence
from typing import Literal, SupportsFloat, get_args

import torch
from torch import Tensor

from diffrast_b200 import _functions as F
from diffrast_b200 import _kernels as K
from diffrast_b200._cache import TensorCache
from diffrast_b200.backends import require_cuda
from diffrast_b200.context import RasterizeContext
from diffrast_b200.topology import TopologyHash, topology_for

FilterMode = Literal["auto", "nearest", "linear", "linear-mipmap-nearest", "linear-mipmap-linear"]
BoundaryMode = Literal["wrap", "clamp", "zero", "cube"]
FILTER_MODES = get_args(FilterMode)
BOUNDARY_MODES = get_args(BoundaryMode)
_MODE_INDEX = {name: i for i, name in enumerate(FILTER_MODES[1:])}
_BOUNDARY_INDEX = {name: i for i, name in enumerate(BOUNDARY_MODES)}

EMPTY_KEY = (1 << 63) - 1


# ---------------------------------------------------------------------------------------------
# rasterize
# ---------------------------------------------------------------------------------------------


def rasterize(
    glctx: RasterizeContext,
    pos: Tensor,
    tri: Tensor,
    resolution: tuple[int, int],
    ranges: Tensor | None = None,
    grad_db: bool = True,
) -> tuple[Tensor, Tensor]:
    """Rasterize triangles into per-pixel barycentrics, depth and triangle ids.

    ``pos`` of shape ``[batch, vertices, 4]`` draws every triangle in every view (instanced mode);
    ``[vertices, 4]`` with ``ranges`` draws ``tri[start : start + count]`` in item ``i`` (range
    mode). Returns ``(rast, rast_db)`` of shape ``[batch, height, width, 4]``: ``(u, v, z / w,
    triangle_id + 1)``, zeros where empty, and ``(du/dx, du/dy, dv/dx, dv/dy)``. A pixel centre
    on an edge belongs to the triangle whose interior lies in +x (+y for a horizontal edge);
    zero-area triangles and triangles with non-finite vertices are not drawn. Coverage is
    identical to diffrast's reference backend.
    """
    resolution = check_rasterize_inputs(glctx, pos, tri, resolution, ranges)
    output_db = getattr(glctx, "output_db", True)
    grad_db = grad_db and output_db
    table = _range_table(ranges, pos.device) if pos.ndim == 2 else None
    rast, rast_db, _ = rasterize_layer(pos, tri, resolution, grad_db, None, table)
    return rast, (rast_db if output_db else rast.new_zeros(*rast.shape[:3], 0))


def rasterize_layer(
    pos: Tensor, tri: Tensor, resolution: tuple[int, int], grad_db: bool, previous: Tensor | None,
    ranges: K.RangeTable | None = None,
) -> tuple[Tensor, Tensor, Tensor]:
    """The depth layer behind ``previous`` (packed keys of the layer before, or ``None``).

    ``pos`` is ``[views, V, 4]``, or ``[V, 4]`` with a device range table (range mode: one launch
    draws every item, ids counted from the start of ``tri`` as diffrast ops.py:490-508 does).
    Returns ``(rast, rast_db, keys)``; ``keys`` is the state for the next layer.
    """
    height, width = resolution
    require_cuda(pos.device)
    views = ranges.items if ranges is not None else pos.shape[0]
    drawn = ranges.total if ranges is not None else tri.shape[0] * views
    if drawn == 0:
        empty = pos.new_zeros(views, height, width, 4)
        keys = torch.full((views, height, width), EMPTY_KEY, dtype=torch.int64, device=pos.device)
        return empty, empty.clone(), keys
    port = F.PositionPort(None, {}, pos)
    with torch.cuda.device(pos.device):
        rast, rast_db, keys, sink = F.Rasterize.apply(
            K.aligned(pos if ranges is None else pos[None]), tri.contiguous(), height, width,
            bool(grad_db), previous, ranges, port,
        )
    if sink.requires_grad and ranges is None:
        # An antialias pass over this rast and the same pos hands its position gradient to this
        # rasterization's backward pass, and a lookup of coordinates interpolated from this rast
        # may run that backward pass itself (see _functions.PositionPort).
        port.sink = sink
        rast._dr_pos_port = port
    return rast, rast_db, keys


def check_rasterize_inputs(glctx, pos, tri, resolution, ranges) -> tuple[int, int]:
    """Validate the arguments of :func:`rasterize`; returns ``(height, width)``."""
    range_mode = isinstance(pos, Tensor) and pos.ndim == 2
    _check(pos, "pos", ndim=2 if range_mode else 3, last=4, dtype=torch.float32)
    _check(tri, "tri", ndim=2, last=3, dtype=torch.int32)
    # rast stores triangle_id + 1 as float32, exact only up to 2**24.
    if tri.shape[0] > 1 << 24:
        raise ValueError(
            f"tri has {tri.shape[0]} triangles, but at most 2**24 = {1 << 24} are supported: "
            "rast stores triangle ids as float32, which is exact only up to there."
        )
    _check_devices(pos=pos, tri=tri)
    _check_indices(tri, pos.shape[-2])
    if pos.device != glctx.device:
        raise ValueError(f"pos is on {pos.device} but the context is on {glctx.device}.")
    if range_mode:
        _check_ranges(ranges, tri.shape[0])
    return _check_resolution(resolution)


_range_tables: dict[torch.device, TensorCache[K.RangeTable]] = {}


def _range_table(ranges: Tensor, device: torch.device) -> K.RangeTable:
    """Device table of ``ranges``, made once per tensor object and device (so that a call
    captured into a CUDA graph copies nothing from the host)."""
    cache = _range_tables.get(device)
    if cache is None:
        cache = _range_tables[device] = TensorCache(lambda r: K.range_table(r, device))
    return cache.get(ranges)


def _check_ranges(ranges: Tensor | None, num_tri: int) -> None:
    if ranges is None:
        raise ValueError(
            "ranges is required when pos has shape [vertices, 4] (range mode); give pos a "
            "leading batch dimension to draw all triangles (instanced mode)."
        )
    _check(ranges, "ranges", ndim=2, last=2, dtype=torch.int32)
    for item, (start, count) in enumerate(ranges.tolist()):
        if start < 0 or count < 0 or start + count > num_tri:
            raise ValueError(
                f"ranges[{item}] = (start {start}, count {count}) does not lie within the "
                f"{num_tri} triangles of tri."
            )


# ---------------------------------------------------------------------------------------------
# interpolate
# ---------------------------------------------------------------------------------------------


def interpolate(
    attr: Tensor,
    rast: Tensor,
    tri: Tensor,
    rast_db: Tensor | None = None,
    diff_attrs: Sequence[int] | Literal["all"] | None = None,
) -> tuple[Tensor, Tensor]:
    """Interpolate vertex attributes over the rasterized triangles.

    ``attr`` is ``[batch, vertices, channels]`` or ``[vertices, channels]`` (shared); returns
    ``(out [batch, h, w, channels], out_da [batch, h, w, 2 * len(diff_attrs)])`` with ``(d/dx,
    d/dy)`` per selected channel, empty when ``diff_attrs`` is not set. Ids past the end of
    ``tri`` are background.
    """
    shared = isinstance(attr, Tensor) and attr.ndim == 2
    layout = "[batch, vertices, channels] or [vertices, channels]"
    _check(attr, "attr", ndim=2 if shared else 3, dtype=torch.float32, layout=layout)
    _check(rast, "rast", ndim=4, last=4, dtype=torch.float32)
    _check(tri, "tri", ndim=2, last=3, dtype=torch.int32)
    if attr.ndim == 3 and attr.shape[0] not in (1, rast.shape[0]):
        raise ValueError(
            f"attr batch size {attr.shape[0]} does not match rast batch size {rast.shape[0]}."
        )
    _check_devices(attr=attr, rast=rast, tri=tri, rast_db=rast_db)
    channels = _diff_channels(diff_attrs, attr.shape[-1])
    empty = rast_db is not None and rast_db.ndim == 4 and rast_db.shape[-1] == 0
    if rast_db is not None and not empty:
        _check(rast_db, "rast_db", ndim=4, last=4, dtype=torch.float32)
        if rast_db.shape != rast.shape:
            raise ValueError(
                f"rast_db must have the same shape as rast, got {tuple(rast_db.shape)} and "
                f"{tuple(rast.shape)}."
            )
    if not channels:
        rast_db = None
    elif rast_db is None or empty:
        given = ", but the one given is empty" if empty else ""
        raise ValueError(f"rast_db is required when diff_attrs is set{given}.")
    _check_indices(tri, attr.shape[-2])
    require_cuda(rast.device)
    batch, height, width, _ = rast.shape
    if tri.shape[0] == 0 or rast.numel() == 0:
        out = attr.new_zeros(batch, height, width, attr.shape[-1])
        return out, attr.new_zeros(batch, height, width, 2 * len(channels))
    with torch.cuda.device(rast.device):
        diff = K.diff_table(tuple(channels), rast.device)
        port = F.CoordinatePort(None, {}, tuple(channels))
        out, out_da, sink = F.Interpolate.apply(
            attr, K.aligned(rast), None if rast_db is None else K.aligned(rast_db),
            tri.contiguous(), diff, port,
        )
    if sink.requires_grad:
        # Lookups that read channel slices of out / out_da hand their gradients back through
        # this port instead of through whole gradient images (see _functions.CoordinatePort).
        port.sink = sink
        out._dr_port = port
        out_da._dr_port = port
    return out, out_da


def _diff_channels(diff_attrs, num_channels: int) -> list[int]:
    if diff_attrs is None:
        return []
    expected = f"diff_attrs must be a sequence of channel indices, 'all' or None, got {diff_attrs!r}."
    if isinstance(diff_attrs, str):
        if diff_attrs != "all":
            raise ValueError(expected)
        return list(range(num_channels))
    try:
        channels = [operator.index(c) for c in diff_attrs]
    except TypeError:
        raise TypeError(expected) from None
    if any(c < 0 or c >= num_channels for c in channels):
        raise ValueError(f"diff_attrs {channels} out of range for {num_channels} channels.")
    return channels


# ---------------------------------------------------------------------------------------------
# texture
# ---------------------------------------------------------------------------------------------


class MipStack:
    """Mip levels built by :func:`texture_construct_mip`, passed to :func:`texture` as ``mip``.

    Holds levels 1 and up as tensors (each produced by the mip-build kernel); the base level is
    the texture passed to :func:`texture`.
    """

    __slots__ = ("cube_mode", "levels", "shape")

    def __init__(self, levels: Sequence[Tensor], cube_mode: bool, shape: Sequence[int]) -> None:
        self.levels = tuple(levels)
        self.cube_mode = cube_mode
        self.shape = tuple(shape)


def _chain_length(h: int, w: int, max_mip_level: int | None) -> int:
    """Number of halvings of the full chain, limited by ``max_mip_level`` (reference.py:433-446)."""
    count = 0
    while max(h, w) > 1 and (max_mip_level is None or count < max_mip_level):
        h, w = (h + 1) // 2, (w + 1) // 2
        count += 1
    return count


def _build_chain(tex: Tensor, max_mip_level: int | None) -> list[Tensor]:
    count = _chain_length(tex.shape[-3], tex.shape[-2], max_mip_level)
    if count == 0:
        return []
    require_cuda(tex.device)
    with torch.cuda.device(tex.device):
        return list(F.MipChain.apply(tex.contiguous(), count))


def texture(
    tex: Tensor,
    uv: Tensor,
    uv_da: Tensor | None = None,
    mip_level_bias: Tensor | None = None,
    mip: MipStack | Sequence[Tensor] | None = None,
    filter_mode: FilterMode = "auto",
    boundary_mode: BoundaryMode = "wrap",
    max_mip_level: int | None = None,
) -> Tensor:
    """Sample a 2D texture ``[batch, h, w, C]`` or a cube map ``[batch, 6, s, s, C]``.

    Arguments as in diffrast (``ops.py:139-236``): ``uv`` ``[batch, H, W, 2]`` (directions
    ``[.., 3]`` for a cube), ``uv_da`` ``[.., 4]`` (``[.., 6]``), ``mip_level_bias`` ``[batch, H,
    W]``, ``mip`` a :class:`MipStack` or a list of levels 1.., ``filter_mode`` ``"auto"`` picks
    trilinear when a level of detail is given. Pixels whose coordinates or level are NaN (or
    undefined) are NaN and pass no gradient; invalid cube directions read zero.
    """
    if filter_mode not in FILTER_MODES:
        raise ValueError(f"Unknown filter_mode {filter_mode!r}; expected one of {FILTER_MODES}.")
    if boundary_mode not in BOUNDARY_MODES:
        raise ValueError(
            f"Unknown boundary_mode {boundary_mode!r}; expected one of {BOUNDARY_MODES}."
        )
    cube = boundary_mode == "cube"
    _check_texture(tex, "tex", cube, 'boundary_mode="cube"')
    _check(uv, "uv", ndim=4, last=3 if cube else 2, dtype=torch.float32)
    if tex.shape[0] not in (1, uv.shape[0]):
        raise ValueError(
            f"tex batch size {tex.shape[0]} does not match uv batch size {uv.shape[0]}."
        )
    if isinstance(uv_da, Tensor) and uv_da.ndim == 4 and uv_da.shape[-1] == 0:
        uv_da = None
    has_lod = uv_da is not None or mip_level_bias is not None
    if filter_mode == "auto":
        filter_mode = "linear-mipmap-linear" if has_lod else "linear"
    if "mipmap" in filter_mode and not has_lod:
        raise ValueError(f"filter_mode {filter_mode!r} requires uv_da or mip_level_bias.")
    if uv_da is not None:
        _check(uv_da, "uv_da", ndim=4, last=6 if cube else 4, dtype=torch.float32)
        if uv_da.shape[:3] != uv.shape[:3]:
            raise ValueError("uv_da must match uv in batch, height and width.")
    if mip_level_bias is not None:
        _check(mip_level_bias, "mip_level_bias", ndim=3, dtype=torch.float32)
        if mip_level_bias.shape != uv.shape[:3]:
            raise ValueError("mip_level_bias must match uv in batch, height and width.")
    if max_mip_level is not None and max_mip_level < 0:
        raise ValueError(f"max_mip_level must be non-negative, got {max_mip_level}.")
    given = None if mip is None else _check_mip(mip, tex, cube)
    _check_devices(tex=tex, uv=uv, uv_da=uv_da, mip_level_bias=mip_level_bias)
    require_cuda(uv.device)

    mipmapped = "mipmap" in filter_mode
    mode = _MODE_INDEX[filter_mode]
    if uv.numel() == 0:
        return tex.new_zeros(*uv.shape[:3], tex.shape[-1])
    if mipmapped and given is None:
        # The chain is built inside the lookup's autograd function, whose backward pushes the
        # level gradients down the chain without leaving the kernels' buffers.
        count = _chain_length(tex.shape[-3], tex.shape[-2], max_mip_level)
        if mode < 3:
            uv_da = None if uv_da is None else uv_da.detach()
            mip_level_bias = None if mip_level_bias is None else mip_level_bias.detach()
        uv_src, uv_spec = _channel_slice(uv)
        da_src, da_spec = _channel_slice(uv_da)
        route, sink, uv_src, uv_spec, da_src, da_spec = _route(uv_src, uv_spec, da_src, da_spec,
                                                               _needs_grad(uv_da), cube)
        with torch.cuda.device(uv.device):
            return F.TextureChain.apply(
                uv_src, da_src, None if mip_level_bias is None else mip_level_bias.contiguous(),
                mode, _BOUNDARY_INDEX[boundary_mode], count, tex, uv_spec, da_spec, route, sink,
                _pos_sink(route),
            )
    if mipmapped:
        if given is None:
            levels = [tex, *_build_chain(tex, max_mip_level)]
        else:
            levels = [tex, *given]
            if max_mip_level is not None:
                levels = levels[: max_mip_level + 1]
    else:
        levels = [tex]
    # Inputs the output does not depend on stay out of the graph, as in the reference.
    if mode == 0:
        uv = uv.detach()
    if mode < 3:
        uv_da = None if uv_da is None or mode < 2 else uv_da.detach()
        mip_level_bias = None if mip_level_bias is None or mode < 2 else mip_level_bias.detach()
    # uv and uv_da may be channel slices of a wider tensor (such as interpolate's output): the
    # kernels read them in place through their pixel stride.
    uv_src, uv_spec = _channel_slice(uv)
    da_src, da_spec = _channel_slice(uv_da)
    route, sink, uv_src, uv_spec, da_src, da_spec = _route(uv_src, uv_spec, da_src, da_spec,
                                                           _needs_grad(uv_da), cube)
    with torch.cuda.device(uv.device):
        return F.Texture.apply(
            uv_src, da_src, None if mip_level_bias is None else mip_level_bias.contiguous(), mode,
            _BOUNDARY_INDEX[boundary_mode], uv_spec, da_spec, route, sink, _pos_sink(route),
            *levels,
        )


def _needs_grad(t: Tensor | None) -> bool:
    return t is not None and t.requires_grad and torch.is_grad_enabled()


def _route(uv_src, uv_spec, da_src, da_spec, has_da: bool, cube: bool = False):
    """``(route, sink, uv_src, uv_spec, da_src, da_spec)`` for a lookup whose uv (and uv_da, if
    given) are the outputs of one :func:`interpolate` call or channel slices of them: its
    coordinate gradients then go back through that call's port, and uv_src / da_src enter the
    lookup detached (a whole output counts as the slice of all its channels). ``(None, None,
    uv_src, uv_spec, da_src, da_spec)`` otherwise."""
    unrouted = None, None, uv_src, uv_spec, da_src, da_spec
    port = getattr(uv_src, "_dr_port", None)
    if port is None or not (uv_spec is not None or _needs_grad(uv_src)):
        return unrouted
    if has_da and (getattr(da_src, "_dr_port", None) is not port
                   or not (da_spec is not None or _needs_grad(da_src))):
        return unrouted
    if uv_spec is None:
        uv_spec = (0, uv_src.shape[-1])
    if has_da and da_spec is None:
        da_spec = (0, da_src.shape[-1])
    # A 2D lookup of coordinates interpolated from rasterize's own rast also depends on that
    # rasterization's sink, so that its backward pass may run the rasterizer's backward pass
    # (the rasterizer's backward pass then collects the position gradient it leaves).
    pos_port = None
    geometry = port.geometry.tensors() if port.geometry is not None and not cube else None
    if geometry is not None:
        candidate = getattr(geometry[1], "_dr_pos_port", None)
        if candidate is not None and candidate.sink is not None and candidate.sink.requires_grad:
            pos_port = candidate
    route = F.Route(port.pending, want_uv=True, want_da=has_da, port=port, pos_port=pos_port)
    return (route, port.sink, uv_src.detach(), uv_spec,
            None if da_src is None else da_src.detach(), da_spec)


def _pos_sink(route) -> Tensor | None:
    return None if route is None or route.pos_port is None else route.pos_port.sink



def _channel_slice(t: Tensor | None):
    """``(base, (first channel, count))`` when ``t`` is a slice of the last dimension of a
    contiguous tensor and gradients flow to it (interpolate's ``out[..., 0:2]``, say), so that
    the lookup can write its gradient straight into the base's; ``(t, None)`` otherwise."""
    if t is None or not t.requires_grad or not torch.is_grad_enabled():
        return t, None
    base = t._base
    if (base is None or not base.requires_grad or base.ndim != t.ndim or base.dtype != t.dtype
            or not base.is_contiguous() or base.shape[:-1] != t.shape[:-1]
            or t.stride()[:-1] != base.stride()[:-1] or t.stride(-1) != 1):
        return t, None
    first = t.storage_offset() - base.storage_offset()
    if first < 0 or first + t.shape[-1] > base.shape[-1]:
        return t, None
    return base, (first, t.shape[-1])


def texture_construct_mip(
    tex: Tensor, max_mip_level: int | None = None, cube_mode: bool = False
) -> MipStack:
    """Build mip levels 1.. of ``tex`` once, for several :func:`texture` calls.

    Gradients flow from the levels back to ``tex`` if it requires them (rebuild after ``tex``
    changes). ``cube_mode`` must be true for a cube map.
    """
    _check_texture(tex, "tex", cube_mode, "cube_mode=True")
    if max_mip_level is not None and max_mip_level < 0:
        raise ValueError(f"max_mip_level must be non-negative, got {max_mip_level}.")
    return MipStack(_build_chain(tex, max_mip_level), bool(cube_mode), tex.shape)


def _check_texture(t: Tensor, name: str, cube: bool, cube_option: str) -> None:
    if isinstance(t, Tensor) and t.ndim == 5 and not cube:
        raise ValueError(
            f"{name} has the shape of a cube map, {tuple(t.shape)}, which needs {cube_option}."
        )
    if isinstance(t, Tensor) and t.ndim == 4 and cube:
        raise ValueError(
            f"{cube_option} needs {name} to be a cube map of shape "
            f"[batch, 6, size, size, channels], got {tuple(t.shape)}."
        )
    _check(t, name, ndim=5 if cube else 4, dtype=torch.float32)
    if cube and (t.shape[1] != 6 or t.shape[2] != t.shape[3]):
        raise ValueError(
            f"{name} must have six square faces, [batch, 6, size, size, channels], "
            f"got {tuple(t.shape)}."
        )
    if 0 in t.shape[1:]:
        raise ValueError(
            f"{name} must have at least one texel and one channel, got shape {tuple(t.shape)}."
        )


def _check_mip(mip, tex: Tensor, cube: bool) -> list[Tensor]:
    if isinstance(mip, MipStack):
        if mip.cube_mode != cube:
            raise ValueError(
                f"mip was constructed with cube_mode={mip.cube_mode}, which does not match "
                f"{'a cube map' if cube else 'a 2D texture'}."
            )
        if mip.shape != tuple(tex.shape):
            raise ValueError(
                f"mip was constructed for a texture of shape {mip.shape}, but tex has shape "
                f"{tuple(tex.shape)}."
            )
        levels = list(mip.levels)
    elif isinstance(mip, Sequence):
        levels = list(mip)
    else:
        raise TypeError(
            "mip must be a list of tensors or the result of texture_construct_mip, "
            f"got {type(mip).__name__}."
        )
    for index, level in enumerate(levels, start=1):
        name = f"mip level {index}"
        _check_texture(level, name, cube, 'boundary_mode="cube"')
        if level.shape[-1] != tex.shape[-1]:
            raise ValueError(f"{name} has {level.shape[-1]} channels but tex has {tex.shape[-1]}.")
        if level.shape[0] not in (1, tex.shape[0]):
            raise ValueError(
                f"{name} has batch size {level.shape[0]}; expected 1 or that of tex, "
                f"{tex.shape[0]}."
            )
        if level.device != tex.device:
            raise ValueError(f"{name} is on {level.device} but tex is on {tex.device}.")
    return levels


# ---------------------------------------------------------------------------------------------
# antialias
# ---------------------------------------------------------------------------------------------


def antialias(
    color: Tensor,
    rast: Tensor,
    pos: Tensor,
    tri: Tensor,
    topology_hash: TopologyHash | None = None,
    pos_gradient_boost: float = 1.0,
) -> Tensor:
    """Antialias silhouette edges so that visibility changes produce gradients in ``pos``.

    ``color`` ``[batch, h, w, C]``, ``rast`` from :func:`rasterize`, ``pos`` ``[batch, V, 4]``
    or ``[V, 4]`` (shared), ``tri`` the position indices. The edge adjacency of ``tri`` comes from
    ``topology_hash`` or is built on the first call and cached per tensor object.
    """
    topology = _check_antialias_inputs(color, rast, pos, tri, topology_hash, pos_gradient_boost)
    if tri.shape[0] == 0 or color.numel() == 0:
        return color.clone()
    route, sink, pos = _position_route(rast, pos)
    with torch.cuda.device(color.device):
        return F.Antialias.apply(
            color.contiguous(), K.aligned(rast.detach()), K.aligned(pos), tri.contiguous(),
            topology.opposite(tri), float(pos_gradient_boost), route, sink,
        )


def _position_route(rast: Tensor, pos: Tensor):
    """``(route, sink, pos)`` for an antialias pass over ``rast`` from :func:`rasterize` with the
    very ``pos`` tensor it was rasterized from: the position gradient then goes to the
    rasterizer's backward pass and ``pos`` enters detached. ``(None, None, pos)`` otherwise."""
    port = getattr(rast, "_dr_pos_port", None)
    if port is None or port.pos() is not pos or pos.ndim != 3 or not _needs_grad(pos):
        return None, None, pos
    return port.pending, port.sink, pos.detach()


def antialias_mse(
    color: Tensor,
    rast: Tensor,
    pos: Tensor,
    tri: Tensor,
    target: Tensor,
    topology_hash: TopologyHash | None = None,
    pos_gradient_boost: float = 1.0,
    scale: float | None = None,
) -> tuple[Tensor, Tensor]:
    """:func:`antialias` followed by the squared-error loss against ``target``, fused.

    Returns ``(image, loss)``: ``image`` equals ``antialias(color, rast, pos, tri, ...)`` and
    ``loss`` is ``scale * ((image - target) ** 2).sum()``, a 0-dim tensor; ``scale`` defaults to
    ``1 / image.numel()`` (``torch.nn.functional.mse_loss``'s mean). The loss is summed inside the
    antialias kernel and its backward pass forms the image's gradient on the fly, so no loss
    kernels run and no gradient image is stored; gradients reaching ``image`` from elsewhere are
    added. Not part of diffrast's API: a fit that ends in an MSE can call this in place of
    ``antialias`` plus ``mse_loss``.
    """
    _check(color, "color", ndim=4, dtype=torch.float32)
    _check(target, "target", ndim=4, dtype=torch.float32, layout="[batch, height, width, channels]")
    if target.shape != color.shape:
        raise ValueError(f"target must match color, got {tuple(target.shape)} and {tuple(color.shape)}.")
    _check_devices(color=color, target=target)
    if scale is None:
        scale = 1.0 / max(1, color.numel())
    if not isinstance(scale, SupportsFloat):
        raise TypeError(f"scale must be a number, got {scale!r}.")
    topology = _check_antialias_inputs(color, rast, pos, tri, topology_hash, pos_gradient_boost)
    if color.numel() == 0:
        return color.clone(), color.new_zeros(()) + 0.0 * color.sum()
    opposite = topology.opposite(tri) if topology is not None else tri.new_zeros(0)
    route, sink, pos = _position_route(rast, pos)
    with torch.cuda.device(color.device):
        return F.AntialiasMSE.apply(
            color.contiguous(), K.aligned(rast.detach()), K.aligned(pos), tri.contiguous(),
            opposite, target.detach().contiguous(), float(scale), float(pos_gradient_boost),
            route, sink,
        )


def _check_antialias_inputs(color, rast, pos, tri, topology_hash, pos_gradient_boost):
    """Validate the arguments of :func:`antialias`; returns the topology (None without
    triangles)."""
    _check(color, "color", ndim=4, dtype=torch.float32)
    _check(rast, "rast", ndim=4, last=4, dtype=torch.float32)
    shared = isinstance(pos, Tensor) and pos.ndim == 2
    layout = "[batch, vertices, 4] or [vertices, 4]"
    _check(pos, "pos", ndim=2 if shared else 3, last=4, dtype=torch.float32, layout=layout)
    _check(tri, "tri", ndim=2, last=3, dtype=torch.int32)
    if color.shape[:3] != rast.shape[:3]:
        raise ValueError(
            "color must match rast in batch, height and width, got "
            f"{tuple(color.shape)} and {tuple(rast.shape)}."
        )
    if not shared and pos.shape[0] != rast.shape[0]:
        raise ValueError(
            f"pos batch size {pos.shape[0]} does not match rast batch size {rast.shape[0]}."
        )
    if not isinstance(pos_gradient_boost, SupportsFloat):
        raise TypeError(f"pos_gradient_boost must be a number, got {pos_gradient_boost!r}.")
    _check_devices(color=color, rast=rast, pos=pos, tri=tri)
    _check_indices(tri, pos.shape[-2])
    require_cuda(color.device)
    if topology_hash is not None or tri.shape[0]:
        return topology_for(tri, topology_hash)
    return None


def antialias_construct_topology_hash(tri: Tensor) -> TopologyHash:
    """Edge adjacency of ``tri`` for :func:`antialias` (built on the GPU, no sort)."""
    _check(tri, "tri", ndim=2, last=3, dtype=torch.int32)
    return TopologyHash(tri)


# ---------------------------------------------------------------------------------------------
# world-to-clip transform
# ---------------------------------------------------------------------------------------------


def lambert(color: Tensor, normal: Tensor, light_dir: Tensor, ambient: float = 0.0) -> Tensor:
    """Shade ``color`` by the interpolated ``normal`` under a directional light, in one pass.

    Returns ``color * (ambient + max(0, n . l))`` with ``n`` the unit normal of each pixel and
    ``l`` the unit light direction: ``color`` is ``[batch, height, width, channels]``, ``normal``
    ``[batch, height, width, 3]`` (a channel slice of :func:`interpolate`'s output such as
    ``out[..., 2:5]`` is read in place), ``light_dir`` ``[3]`` or ``[batch, 3]`` (normalised here).
    A zero normal (background) gets the ambient term alone. Differentiable in ``color`` and
    ``normal``; the light is a constant. Not part of diffrast's API: the shading that its examples
    write with torch elementwise ops, fused forward and backward.
    """
    _check(color, "color", ndim=4, dtype=torch.float32)
    _check(normal, "normal", ndim=4, last=3, dtype=torch.float32,
           layout="[batch, height, width, 3]")
    if normal.shape[:3] != color.shape[:3]:
        raise ValueError(
            f"normal must match color in batch, height and width, got {tuple(normal.shape)} and "
            f"{tuple(color.shape)}."
        )
    if not isinstance(light_dir, Tensor) or light_dir.dtype != torch.float32:
        raise TypeError("light_dir must be a torch.float32 tensor of shape [3] or [batch, 3].")
    light = light_dir.reshape(1, 3) if light_dir.ndim == 1 else light_dir
    if light.ndim != 2 or light.shape[1] != 3 or light.shape[0] not in (1, color.shape[0]):
        raise ValueError(
            f"light_dir must have shape [3] or [batch, 3], got {tuple(light_dir.shape)}."
        )
    if not isinstance(ambient, SupportsFloat):
        raise TypeError(f"ambient must be a number, got {ambient!r}.")
    if color.shape[0] > 65535:
        raise ValueError(f"lambert takes at most 65535 views, got {color.shape[0]}.")
    _check_devices(color=color, normal=normal, light_dir=light_dir)
    require_cuda(color.device)
    if color.numel() == 0:
        return color.clone()
    with torch.cuda.device(color.device):
        return F.Lambert.apply(color.contiguous(), normal, light.detach().contiguous(),
                               float(ambient))


def to_clip(positions: Tensor, matrix: Tensor) -> Tensor:
    """Transform ``[vertices, 3]`` positions by ``[batch, 4, 4]`` matrices to clip space.

    Returns ``[batch, vertices, 4]``, the homogeneous positions ``(x, y, z, 1)`` times the
    transposed matrices, as diffrast's examples compute it with a matmul (examples/common.py:
    320-323); differentiable in both inputs. One shared vertex buffer seen by many cameras thus
    gets a single gradient, summed over the views (and ready for an all-reduce across ranks).
    """
    _check(positions, "positions", ndim=2, last=3, dtype=torch.float32, layout="[vertices, 3]")
    _check(matrix, "matrix", ndim=3, dtype=torch.float32, layout="[batch, 4, 4]")
    if matrix.shape[1:] != (4, 4):
        raise ValueError(f"matrix must have shape [batch, 4, 4], got {tuple(matrix.shape)}.")
    _check_devices(positions=positions, matrix=matrix)
    require_cuda(positions.device)
    with torch.cuda.device(positions.device):
        return F.ToClip.apply(positions.contiguous(), matrix.contiguous())


# ---------------------------------------------------------------------------------------------
# validation helpers (messages as in diffrast ops.py:511-638)
# ---------------------------------------------------------------------------------------------

_LAYOUTS = {
    "pos": "[batch, vertices, 4]",
    "tri": "[triangles, 3]",
    "rast": "[batch, height, width, 4]",
    "rast_db": "[batch, height, width, 4]",
    "color": "[batch, height, width, channels]",
    "tex": "[batch, tex_height, tex_width, channels]",
    "uv": "[batch, height, width, 2]",
    "uv_da": "[batch, height, width, 4]",
    "mip_level_bias": "[batch, height, width]",
}


def _check(t, name: str, ndim: int, last: int | None = None, dtype=None, layout: str | None = None):
    if not isinstance(t, Tensor):
        raise TypeError(f"{name} must be a torch.Tensor, got {type(t).__name__}.")
    if t.ndim != ndim or (last is not None and t.shape[-1] != last):
        if layout is None:
            layout = _LAYOUTS.get(name)
            fits = layout is not None and layout.count(",") + 1 == ndim
            if not fits or (last and not layout.endswith(f" {last}]")):
                layout = f"[{', '.join(['...'] * (ndim - 1) + [str(last) if last else '...'])}]"
        hint = ""
        unbatched = t.ndim == ndim - 1 and (last is None or t.shape[-1:] == (last,))
        if unbatched and layout.startswith("[batch") and " or " not in layout:
            hint = f"; add a batch dimension with {name}[None]"
        raise ValueError(f"{name} must have shape {layout}, got {tuple(t.shape)}{hint}.")
    if dtype is not None and t.dtype != dtype:
        cast = {torch.float32: "float", torch.int32: "int"}.get(dtype)
        hint = f"; convert it with {name}.{cast}()" if cast and name.isidentifier() else ""
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}{hint}.")


def _check_devices(**tensors) -> None:
    devices = {}
    for name, t in tensors.items():
        if t is None:
            continue
        if not isinstance(t, Tensor):
            raise TypeError(f"{name} must be a torch.Tensor, got {type(t).__name__}.")
        devices[name] = t.device
    if len(set(devices.values())) > 1:
        listing = ", ".join(f"{name} on {device}" for name, device in devices.items())
        raise ValueError(f"All inputs must be on the same device; got {listing}.")


def _index_range(tri: Tensor) -> tuple[int, int]:
    low, high = torch.stack(tri.aminmax()).tolist()
    return low, high


_index_ranges: TensorCache[tuple[int, int]] = TensorCache(_index_range)


def _check_indices(tri: Tensor, num_vertices: int, name: str = "tri") -> None:
    """Raise ``ValueError`` if ``tri`` refers to a vertex outside ``[0, num_vertices)``; the range
    is computed once per tensor object (one device sync) and cached until it is modified."""
    if tri.numel() == 0:
        return
    low, high = _index_ranges.get(tri)
    if low < 0 or high >= num_vertices:
        index = low if low < 0 else high
        valid = "there are no vertices"
        if num_vertices > 0:
            valid = f"valid indices are 0 to {num_vertices - 1} for {num_vertices} vertices"
        raise ValueError(f"{name} refers to vertex {index}, but {valid}.")


def _check_resolution(resolution) -> tuple[int, int]:
    values = resolution.tolist() if hasattr(resolution, "tolist") else resolution
    try:
        if not isinstance(values, (list, tuple)) or any(isinstance(r, bool) for r in values):
            raise TypeError
        height, width = (operator.index(r) for r in values)
    except (TypeError, ValueError):
        raise ValueError(f"resolution must be (height, width) as two ints, got {resolution!r}.") from None
    if height <= 0 or width <= 0:
        raise ValueError(f"resolution must be positive, got {resolution!r}.")
    return height, width
