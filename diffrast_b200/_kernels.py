"""Tensor-level calls of the C ABI: outputs and scratch come from PyTorch's caching allocator,
launches go to the current CUDA stream of the tensors' device.

Scratch tensors are released when a function returns while its kernels may still be queued; the
caching allocator only hands that memory to later work on the same stream, so this is safe.
"""

from __future__ import annotations

import contextlib
import functools
import os
from ctypes import byref, c_int64
from typing import NamedTuple

import torch
from torch import Tensor

from diffrast_b200 import _native as N

# Optional per-stage timing: when ``timings`` is a dict, every wrapper below records a pair of CUDA
# events around its launches on the current stream, keyed by stage name. bench.py uses this to
# time the dominant kernel inside its timed region.
timings: dict[str, list] | None = None
# With DIFFRAST_B200_NVTX=1 every wrapper's launches are also enclosed in an NVTX range named
# after its stage ("diffrast_b200.<stage>"), for profilers that filter or group by NVTX.
nvtx = os.environ.get("DIFFRAST_B200_NVTX", "0") not in ("", "0")


def timed(name: str):
    label = f"diffrast_b200.{name}"

    def decorate(fn):
        @functools.wraps(fn)
        def wrapper(*args, **kwargs):
            if nvtx:
                torch.cuda.nvtx.range_push(label)
            try:
                if timings is None:
                    return fn(*args, **kwargs)
                start = torch.cuda.Event(enable_timing=True)
                end = torch.cuda.Event(enable_timing=True)
                start.record()
                out = fn(*args, **kwargs)
                end.record()
                timings.setdefault(name, []).append((start, end))
                return out
            finally:
                if nvtx:
                    torch.cuda.nvtx.range_pop()

        return wrapper

    return decorate


@contextlib.contextmanager
def record_timings():
    """Collect stage timings inside the block; yields the dict of event pairs."""
    global timings
    timings = {}
    try:
        yield timings
    finally:
        timings = None


# Binned-triangle capacity of the rasterizer's setup list, remembered per problem shape so that
# the list is sized right from the second call on.
_capacity: dict[tuple, int] = {}
# Binned-triangle and pair capacities for calls captured into a CUDA graph (which cannot read the
# counts back): twice the largest counts seen by eager calls of the same shape, plus slack.
_graph_capacity: dict[tuple, tuple[int, int]] = {}
# Per device: a word that captured visibility passes set when their counts exceeded those
# capacities (see RasterizeContext.capture_overflowed).
_overflow: dict[torch.device, Tensor] = {}
# The occlusion pass (small triangles facing away set aside, drawn after the rest unless hidden
# everywhere) is used from this many (view, triangle) items per 16 x 16 tile on; either way the
# keys are the same. It is off by default: on config 5 it skips 70% of the set-aside triangles but
# costs more than it saves (8 views: 0.73 + 0.04 + 0.31 ms against 0.83 ms for one pass), since
# the survivors repeat their setup in sparsely filled warps and the set-aside list shares one
# counter.
occlusion_min_items_per_tile = float("inf")


def overflow_word(device: torch.device) -> Tensor:
    word = _overflow.get(device)
    if word is None:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError(
                "diffrast_b200: run rasterize once without CUDA graph capture before capturing it "
                "(the captured call reuses capacities measured by an eager call)."
            )
        word = torch.zeros(1, dtype=torch.int64, device=device)
        _overflow[device] = word
    return word


def aligned(t: Tensor) -> Tensor:
    """Contiguous and 16-byte aligned (rows of four floats are read as float4)."""
    t = t.contiguous()
    if t.data_ptr() % 16:
        t = t.clone()
    return t


def zeros(shape, device: torch.device) -> Tensor:
    """A float32 tensor of zeros made with one device memset on the current stream (the
    gradient buffers the backward scatters accumulate into)."""
    t = torch.empty(shape, dtype=torch.float32, device=device)
    if t.numel():
        N.check(N.lib().dr_zero(t.data_ptr(), t.numel() * 4, N.stream(device)), "dr_zero")
    return t


def zeros_like(t: Tensor) -> Tensor:
    return zeros(t.shape, t.device)


def _scratch(nbytes: int, device: torch.device) -> Tensor:
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


class RangeTable(NamedTuple):
    """Range mode on the device: item ``i`` draws triangles ``start[i] .. start[i] + count``,
    whose flat indices are ``first[i] .. first[i] + count - 1`` (exclusive prefix sums of the
    counts, int64); ``total`` is the sum of the counts."""

    start: Tensor
    first: Tensor
    total: int

    @property
    def items(self) -> int:
        return self.start.shape[0]


def range_table(ranges: Tensor, device: torch.device) -> RangeTable:
    """Device table of a validated ``ranges`` ``[items, 2]`` int32 (start, count)."""
    host = ranges.detach().cpu().to(torch.int64)
    first = torch.zeros(host.shape[0], dtype=torch.int64)
    if host.shape[0] > 1:
        first[1:] = torch.cumsum(host[:-1, 1], 0)
    total = int(host[:, 1].sum()) if host.shape[0] else 0
    return RangeTable(host[:, 0].to(torch.int32).to(device), first.to(device), total)


@timed("raster_visibility")
def raster_keys(pos: Tensor, tri: Tensor, height: int, width: int, prev_keys: Tensor | None,
                ranges: RangeTable | None = None) -> Tensor:
    """Packed visibility keys ``[views, height, width]`` int64 of the nearest layer behind
    ``prev_keys`` (all layers when ``None``). ``pos`` is ``[views, V, 4]``, or ``[1, V, 4]``
    shared by every view; with ``ranges`` the views are its items."""
    lib, dev = N.lib(), pos.device
    s = N.stream(dev)
    pos_batch, num_vert, num_tri = pos.shape[0], pos.shape[1], tri.shape[0]
    batch = ranges.items if ranges is not None else pos_batch
    total = ranges.total if ranges is not None else batch * num_tri
    keys = torch.empty((batch, height, width), dtype=torch.int64, device=dev)
    shape_key = (dev, batch, total, height, width)
    cap = _capacity.get(shape_key, max(1024, min(total, 1 << 16)))
    rs, rf = (N.ptr(ranges.start), N.ptr(ranges.first)) if ranges is not None else (None, None)
    tiles = batch * ((height + 15) // 16) * ((width + 15) // 16)
    occl = None
    if total >= occlusion_min_items_per_tile * max(1, tiles):
        occl = _scratch(lib.dr_raster_occlusion_workspace_bytes(total, batch, height, width), dev)
    occl_ptr, occl_bytes = (occl.data_ptr(), occl.numel()) if occl is not None else (None, 0)

    def setup(cap):
        ws = _scratch(lib.dr_raster_setup_workspace_bytes(cap, height, width), dev)
        N.check(
            lib.dr_raster_setup(pos.data_ptr(), pos_batch, tri.data_ptr(), batch, num_vert,
                                num_tri, rs, rf, total, height, width, N.ptr(prev_keys),
                                keys.data_ptr(), ws.data_ptr(), ws.numel(), cap, occl_ptr,
                                occl_bytes, s),
            "dr_raster_setup",
        )  # fmt: skip
        return ws

    def occluded(setup_ws):
        if occl is None:
            return
        N.check(
            lib.dr_raster_occluded(pos.data_ptr(), pos_batch, tri.data_ptr(), batch, num_vert,
                                   num_tri, rs, rf, total, height, width, N.ptr(prev_keys),
                                   keys.data_ptr(), setup_ws.data_ptr(), occl_ptr, occl_bytes, s),
            "dr_raster_occluded",
        )  # fmt: skip

    if torch.cuda.is_current_stream_capturing():
        # No host round trip: the counts stay on the device, bounded by capacities measured by
        # eager calls; an overflow is flagged on the device.
        word = overflow_word(dev)
        caps = _graph_capacity.get(shape_key)
        if caps is None:
            raise RuntimeError(
                "diffrast_b200: run rasterize once without CUDA graph capture on the same shapes "
                "before capturing it (the captured call reuses capacities measured eagerly)."
            )
        cap, pair_cap = caps
        ws = setup(cap)
        bws = _scratch(lib.dr_raster_bin_workspace_bytes(batch, height, width, pair_cap), dev)
        N.check(
            lib.dr_raster_tiles_device(pos.data_ptr(), pos_batch, tri.data_ptr(), batch, num_vert,
                                       num_tri, height, width, N.ptr(prev_keys), keys.data_ptr(),
                                       ws.data_ptr(), cap, pair_cap, bws.data_ptr(), bws.numel(),
                                       word.data_ptr(), s),
            "dr_raster_tiles_device",
        )  # fmt: skip
        occluded(ws)
        # While the device's overflow word is set, the keys are poisoned (NaN downstream).
        N.check(lib.dr_raster_poison_keys(word.data_ptr(), keys.data_ptr(), keys.numel(), s),
                "dr_raster_poison_keys")
        return keys
    overflow_word(dev)
    binned, pairs = c_int64(0), c_int64(0)
    for _ in range(2):
        ws = setup(cap)
        N.check(lib.dr_raster_counts(ws.data_ptr(), byref(binned), byref(pairs), s), "dr_raster_counts")
        if binned.value <= cap:
            break
        # The list overflowed: rerun with room for every binned triangle (the direct writes of
        # the first run are repeated; they are idempotent minima).
        cap = binned.value + binned.value // 4
        _capacity[shape_key] = cap
    if binned.value > cap:
        raise RuntimeError("diffrast_b200: binned triangle count changed between identical runs")
    old_caps = _graph_capacity.get(shape_key, (0, 0))
    _graph_capacity[shape_key] = (max(old_caps[0], 2 * binned.value + 1024),
                                  max(old_caps[1], 2 * pairs.value + 4096))
    if binned.value > 0 and pairs.value > 0:
        bws = _scratch(lib.dr_raster_bin_workspace_bytes(batch, height, width, pairs.value), dev)
        N.check(
            lib.dr_raster_tiles(pos.data_ptr(), pos_batch, tri.data_ptr(), batch, num_vert,
                                num_tri, height, width, N.ptr(prev_keys), keys.data_ptr(),
                                ws.data_ptr(), binned.value, pairs.value, bws.data_ptr(),
                                bws.numel(), s),
            "dr_raster_tiles",
        )  # fmt: skip
    occluded(ws)
    return keys


@timed("resolve_fwd")
def resolve_fwd(pos: Tensor, tri: Tensor, keys: Tensor) -> tuple[Tensor, Tensor]:
    batch, height, width = keys.shape
    rast = torch.empty((batch, height, width, 4), dtype=torch.float32, device=pos.device)
    rast_db = torch.empty_like(rast)
    N.check(
        N.lib().dr_raster_resolve_fwd(pos.data_ptr(), pos.shape[0], tri.data_ptr(),
                                      keys.data_ptr(), batch, pos.shape[1], tri.shape[0], height,
                                      width, rast.data_ptr(), rast_db.data_ptr(),
                                      N.stream(pos.device)),
        "dr_raster_resolve_fwd",
    )  # fmt: skip
    return rast, rast_db


@timed("resolve_bwd")
def resolve_bwd(pos: Tensor, tri: Tensor, keys: Tensor, grad_rast: Tensor,
                grad_db: Tensor | None, start: Tensor | None = None) -> Tensor:
    """Position gradient of rast / rast_db, accumulated into ``start`` (a gradient of pos's
    shape that other ops produced, updated in place) or into zeros."""
    batch, height, width = keys.shape
    if start is not None and start.shape == pos.shape and start.is_contiguous():
        grad_pos = start
    else:
        grad_pos = zeros_like(pos) if start is None else start.reshape(pos.shape).clone()
    N.check(
        N.lib().dr_raster_resolve_bwd(pos.data_ptr(), pos.shape[0], tri.data_ptr(),
                                      keys.data_ptr(), batch, pos.shape[1], tri.shape[0], height,
                                      width, grad_rast.data_ptr(), N.ptr(grad_db),
                                      grad_pos.data_ptr(), N.stream(pos.device)),
        "dr_raster_resolve_bwd",
    )  # fmt: skip
    return grad_pos


_diff_tables: dict[tuple, Tensor] = {}


def diff_table(channels: tuple[int, ...], device: torch.device) -> Tensor | None:
    """Device copy of the ``diff_attrs`` channel list, made once per list and device."""
    if not channels:
        return None
    key = (channels, device)
    table = _diff_tables.get(key)
    if table is None:
        table = torch.tensor(channels, dtype=torch.int32, device=device)
        _diff_tables[key] = table
    return table


def padded_rows(attr3: Tensor) -> tuple[Tensor, int]:
    """``attr3`` with its vertex rows padded to a multiple of 4 floats when that lets the kernels
    read them with 16-byte loads (at most 8 channels), and the row stride."""
    channels = attr3.shape[2]
    stride = (channels + 3) // 4 * 4
    if stride == channels or channels > 8:
        return attr3, channels
    return torch.nn.functional.pad(attr3, (0, stride - channels)), stride


@timed("interpolate_fwd")
def interpolate_fwd(attr3: Tensor, rast: Tensor, rast_db: Tensor | None, tri: Tensor,
                    diff: Tensor | None, channels: int | None = None) -> tuple[Tensor, Tensor]:
    """``attr3`` ``[attr_batch, V, S]``: rows of S floats whose first ``channels`` (default S) are
    the attributes (S > channels for rows padded by :func:`padded_rows`)."""
    batch, height, width, _ = rast.shape
    attr_stride = attr3.shape[2]
    channels = attr_stride if channels is None else channels
    num_diff = 0 if diff is None else diff.shape[0]
    out = torch.empty((batch, height, width, channels), dtype=torch.float32, device=rast.device)
    out_da = torch.empty((batch, height, width, 2 * num_diff), dtype=torch.float32, device=rast.device)
    N.check(
        N.lib().dr_interpolate_fwd(attr3.data_ptr(), attr3.shape[0], attr3.shape[1], channels,
                                   attr_stride, rast.data_ptr(), N.ptr(rast_db), tri.data_ptr(), tri.shape[0],
                                   N.ptr(diff), num_diff, batch, height, width, out.data_ptr(),
                                   out_da.data_ptr(), N.stream(rast.device)),
        "dr_interpolate_fwd",
    )  # fmt: skip
    return out, out_da


@timed("interpolate_bwd")
def interpolate_bwd(attr3, rast, rast_db, tri, diff, grad_out, grad_out_da, need_attr,
                    part=None, part_first=0, part_da=None, da_first=0):
    """Gradients of attr (``attr3`` unpadded, ``[attr_batch, V, channels]``), rast and rast_db.

    ``grad_out`` / ``grad_out_da`` are whole gradient images or None; ``part`` (``[batch, h, w,
    k]``, contiguous) adds the gradient of out channels ``part_first ..``, ``part_da`` that of
    out_da channels ``da_first ..``."""
    batch, height, width, _ = rast.shape
    channels = attr3.shape[2]
    num_diff = 0 if diff is None else diff.shape[0]
    grad_attr = zeros_like(attr3) if need_attr else None
    grad_rast = torch.empty_like(rast)
    has_da = grad_out_da is not None or part_da is not None
    grad_db = torch.empty_like(rast) if has_da else None
    lib = N.lib()
    if part is None and part_da is None:
        if grad_out is None:
            grad_out = torch.zeros((*rast.shape[:3], channels), device=rast.device)
        status = lib.dr_interpolate_bwd(
            attr3.data_ptr(), attr3.shape[0], attr3.shape[1], channels, rast.data_ptr(),
            N.ptr(rast_db), tri.data_ptr(), tri.shape[0], N.ptr(diff), num_diff, batch, height,
            width, grad_out.data_ptr(), N.ptr(grad_out_da), N.ptr(grad_attr),
            grad_rast.data_ptr(), N.ptr(grad_db), N.stream(rast.device))
        N.check(status, "dr_interpolate_bwd")
    else:
        status = lib.dr_interpolate_bwd_parts(
            attr3.data_ptr(), attr3.shape[0], attr3.shape[1], channels, rast.data_ptr(),
            N.ptr(rast_db), tri.data_ptr(), tri.shape[0], N.ptr(diff), num_diff, batch, height,
            width, N.ptr(grad_out), N.ptr(grad_out_da), N.ptr(part), part_first,
            0 if part is None else part.shape[-1], N.ptr(part_da), da_first,
            0 if part_da is None else part_da.shape[-1], N.ptr(grad_attr), grad_rast.data_ptr(),
            N.ptr(grad_db), N.stream(rast.device))
        N.check(status, "dr_interpolate_bwd_parts")
    return grad_attr, grad_rast, grad_db


def pixel_rows(t: Tensor | None) -> tuple[Tensor | None, int]:
    """``t`` (``[batch, h, w, k]``) with its pixel stride in floats, copied only when its pixels
    are not equally spaced rows of contiguous channels."""
    if t is None:
        return None, 0
    b, h, w, k = t.shape
    sb, sh, sw, sk = t.stride()
    uniform = sk == 1 and (h == 1 or sh == w * sw) and (b == 1 or sb == h * sh) and sw >= k
    if not uniform:
        t = t.contiguous()
        sw = k
    return t, sw


def _pixel_stride(t: Tensor) -> int:
    """Pixel stride of an output view ``[batch, h, w, k]`` whose pixels are equally spaced rows
    of contiguous channels (checked)."""
    b, h, w, k = t.shape
    sb, sh, sw, sk = t.stride()
    if not (sk == 1 and (h == 1 or sh == w * sw) and (b == 1 or sb == h * sh) and sw >= k):
        raise ValueError("gradient output views must have equally spaced pixels")
    return sw


def _level_tables(levels: list[Tensor], cube: bool):
    heights = [lv.shape[-3] for lv in levels]
    widths = [lv.shape[-2] for lv in levels]
    strides = [0 if lv.shape[0] == 1 else lv[0].numel() for lv in levels]
    return N.int32_array(heights), N.int32_array(widths), N.int64_array(strides)


@timed("texture_fwd")
def texture_fwd(levels: list[Tensor], uv: Tensor, uv_da: Tensor | None, bias: Tensor | None,
                mode: int, boundary: int) -> Tensor:
    batch, height, width = uv.shape[:3]
    channels = levels[0].shape[-1]
    out = torch.empty((batch, height, width, channels), dtype=torch.float32, device=uv.device)
    hs, ws, bs = _level_tables(levels, boundary == 3)
    uv, uv_stride = pixel_rows(uv)
    uv_da, da_stride = pixel_rows(uv_da)
    N.check(
        N.lib().dr_texture_fwd(N.pointer_array([lv.data_ptr() for lv in levels]), hs, ws, bs,
                               len(levels), channels, uv.data_ptr(), uv_stride, N.ptr(uv_da),
                               da_stride, N.ptr(bias), batch, height, width, mode, boundary,
                               out.data_ptr(), N.stream(uv.device)),
        "dr_texture_fwd",
    )  # fmt: skip
    return out


@timed("texture_bwd")
def texture_bwd(levels, uv, uv_da, bias, mode, boundary, grad_out, want_uv, want_da, want_bias,
                keep_padded=False, grad_uv=None, grad_da=None, uv_first=-1, da_first=-1):
    """Level gradients and, as wanted, those of uv, uv_da and the bias. ``grad_uv`` / ``grad_da``
    may be given as outputs: with ``uv_first`` / ``da_first`` = -1 a ``[batch, h, w, k]`` view
    that receives the gradient; with c >= 0 a tensor of wider pixel records (``[batch, h, w, K]``)
    whose channels c.. receive it and whose other channels are set to zero."""
    batch, height, width = uv.shape[:3]
    channels = levels[0].shape[-1]
    grads, stride = _level_gradients(levels)
    if want_uv and grad_uv is None:
        grad_uv = torch.empty(uv.shape, dtype=torch.float32, device=uv.device)
    if want_da and grad_da is None:
        grad_da = torch.empty(uv_da.shape, dtype=torch.float32, device=uv.device)
    grad_uv = grad_uv if want_uv else None
    grad_da = grad_da if want_da else None
    guv_stride = 0 if grad_uv is None else _pixel_stride(grad_uv)
    gda_stride = 0 if grad_da is None else _pixel_stride(grad_da)
    uv_first = uv_first if grad_uv is not None else -1
    da_first = da_first if grad_da is not None else -1
    uv, uv_stride = pixel_rows(uv)
    uv_da, da_stride = pixel_rows(uv_da)
    grad_bias = torch.empty_like(bias) if want_bias else None
    hs, ws, bs = _level_tables(levels, boundary == 3)
    N.check(
        N.lib().dr_texture_bwd(N.pointer_array([lv.data_ptr() for lv in levels]),
                               N.pointer_array([g.data_ptr() for g in grads]), hs, ws, bs,
                               len(levels), channels, stride, uv.data_ptr(), uv_stride,
                               N.ptr(uv_da), da_stride, N.ptr(bias),
                               batch, height, width, mode, boundary, grad_out.data_ptr(),
                               N.ptr(grad_uv), guv_stride, uv_first, N.ptr(grad_da),
                               gda_stride, da_first, N.ptr(grad_bias), N.stream(uv.device)),
        "dr_texture_bwd",
    )  # fmt: skip
    if stride != channels and not keep_padded:
        grads = [g[..., :channels].contiguous() for g in grads]
    return grads, grad_uv, grad_da, grad_bias


@timed("texture_chain")
def texture_chain_bwd(g_uv: Tensor, g_da: Tensor | None, want_da: bool, chain) -> None:
    """The chained position part of a lookup on its own (``dr_texture_chain_bwd``): from its
    compact coordinate gradients, the interpolation's and the rasterizer's backward passes,
    accumulated into ``chain.raster.grad_pos``."""
    batch, height, width = g_uv.shape[:3]
    r = chain.raster
    attr = chain.attr
    N.check(
        N.lib().dr_texture_chain_bwd(
            g_uv.contiguous().data_ptr(), N.ptr(g_da.contiguous() if g_da is not None else None),
            batch, height, width, chain.tri.data_ptr(), chain.tri.shape[0], attr.data_ptr(),
            attr.shape[0], attr.shape[1], attr.shape[2], chain.cu, chain.cv, chain.du, chain.dv,
            r.keys.data_ptr(), r.pos.data_ptr(), r.pos.shape[0], r.pos.shape[1],
            int(r.grad_db and want_da and g_da is not None), r.grad_pos.data_ptr(),
            N.stream(g_uv.device)),
        "dr_texture_chain_bwd",
    )  # fmt: skip


def _level_gradients(levels):
    """Zeroed gradient buffers of all levels and their channel stride. Three-channel gradients
    are accumulated in four-channel buffers, so that each texel takes one 16-byte vector
    reduction (the caller drops the padding). One buffer (one memset) holds all levels; each
    level's part is a multiple of 16 bytes long when the stride is 4, so every level stays
    aligned for vector reductions."""
    channels = levels[0].shape[-1]
    stride = 4 if channels == 3 else channels
    sizes = [lv[..., 0].numel() * stride for lv in levels]
    flat = zeros(sum(sizes), levels[0].device)
    grads, at = [], 0
    for lv, size in zip(levels, sizes):
        grads.append(flat[at:at + size].view(*lv.shape[:-1], stride))
        at += size
    return grads, stride


@timed("texture_bwd")
def texture_bwd_chained(levels, uv, uv_da, bias, mode, boundary, grad_out, want_da, want_bias,
                        chain, keep_padded=False):
    """Texture backward with the interpolation's backward for the coordinates fused in
    (``dr_texture_bwd_interp``): level gradients, the bias gradient as wanted, and in place of
    the coordinate gradients ``(grad_rast, grad_db)`` of the interpolation ``chain`` that made uv
    and uv_da (``grad_db`` None unless ``want_da``). With ``chain.raster`` the rasterizer's
    backward pass runs too (``dr_texture_bwd_resolve``): the position gradient is accumulated
    into ``chain.raster.grad_pos`` and ``(None, None)`` stand for rast's and rast_db's."""
    batch, height, width = uv.shape[:3]
    channels = levels[0].shape[-1]
    grads, stride = _level_gradients(levels)
    rast = chain.rast
    uv, uv_stride = pixel_rows(uv)
    uv_da, da_stride = pixel_rows(uv_da)
    grad_bias = torch.empty_like(bias) if want_bias else None
    hs, ws, bs = _level_tables(levels, boundary == 3)
    attr = chain.attr
    common = (N.pointer_array([lv.data_ptr() for lv in levels]),
              N.pointer_array([g.data_ptr() for g in grads]), hs, ws, bs, len(levels), channels,
              stride, uv.data_ptr(), uv_stride, N.ptr(uv_da), da_stride, N.ptr(bias), batch,
              height, width, mode, boundary, grad_out.data_ptr(), N.ptr(grad_bias),
              rast.data_ptr(), chain.tri.data_ptr(), chain.tri.shape[0], attr.data_ptr(),
              attr.shape[0], attr.shape[1], attr.shape[2], chain.cu, chain.cv, chain.du,
              chain.dv)  # fmt: skip
    grad_rast = grad_db = None
    if chain.raster is None:
        grad_rast = torch.empty(rast.shape, dtype=torch.float32, device=rast.device)
        grad_db = torch.empty(rast.shape, dtype=torch.float32, device=rast.device) if want_da else None
        N.check(N.lib().dr_texture_bwd_interp(*common, grad_rast.data_ptr(), N.ptr(grad_db),
                                              N.stream(uv.device)), "dr_texture_bwd_interp")
    else:
        r = chain.raster
        pos = r.pos
        N.check(N.lib().dr_texture_bwd_resolve(*common, r.keys.data_ptr(), pos.data_ptr(),
                                               pos.shape[0], pos.shape[1],
                                               int(r.grad_db and want_da), r.grad_pos.data_ptr(),
                                               N.stream(uv.device)), "dr_texture_bwd_resolve")
    if stride != channels and not keep_padded:
        grads = [g[..., :channels].contiguous() for g in grads]
    return grads, grad_rast, grad_db, grad_bias


def _images(level: Tensor) -> int:
    return level.shape[0] * (6 if level.ndim == 5 else 1)


@timed("mip_build")
def mip_down(level: Tensor) -> Tensor:
    h, w, c = level.shape[-3], level.shape[-2], level.shape[-1]
    out = torch.empty((*level.shape[:-3], (h + 1) // 2, (w + 1) // 2, c), dtype=torch.float32,
                      device=level.device)
    N.check(N.lib().dr_mip_downsample(level.data_ptr(), _images(level), h, w, c, out.data_ptr(),
                                      N.stream(level.device)), "dr_mip_downsample")  # fmt: skip
    return out


@timed("mip_build")
def mip_build(tex: Tensor, count: int) -> list[Tensor]:
    """Levels 1 .. count of ``tex`` (``[.., h, w, C]``, contiguous), each its own tensor, made by
    ``dr_mip_build`` (runs of even halvings several levels per launch)."""
    h, w, c = tex.shape[-3], tex.shape[-2], tex.shape[-1]
    levels, lh, lw = [], h, w
    for _ in range(count):
        lh, lw = (lh + 1) // 2, (lw + 1) // 2
        levels.append(torch.empty((*tex.shape[:-3], lh, lw, c), dtype=torch.float32,
                                  device=tex.device))
    if count:
        N.check(N.lib().dr_mip_build(tex.data_ptr(), _images(tex), h, w, c, count,
                                     N.pointer_array([lv.data_ptr() for lv in levels]),
                                     N.stream(tex.device)), "dr_mip_build")  # fmt: skip
    return levels


@timed("mip_adjoint")
def mip_build_bwd(grads: list[Tensor], out: Tensor | None = None) -> None:
    """Pushes the gradients of levels 1.. (``grads[1:]``) down into the base gradient
    ``grads[0]`` in place, or, given ``out`` (fewer channels: without the padding), writes the
    base result there instead; the coarser buffers are left in an unspecified state."""
    base = grads[0]
    h, w, c = base.shape[-3], base.shape[-2], base.shape[-1]
    N.check(N.lib().dr_mip_build_bwd(N.pointer_array([g.data_ptr() for g in grads]),
                                     _images(base), h, w, c, len(grads) - 1, N.ptr(out),
                                     0 if out is None else out.shape[-1],
                                     N.stream(base.device)), "dr_mip_build_bwd")  # fmt: skip


@timed("mip_adjoint")
def mip_down_bwd(grad_coarse: Tensor, grad_fine: Tensor, out: Tensor | None = None) -> None:
    """Adds the adjoint of one mip step of ``grad_coarse`` into ``grad_fine`` (in place), or,
    given ``out`` (fewer channels, e.g. without the padding), writes the sum there instead."""
    h, w, c = grad_fine.shape[-3], grad_fine.shape[-2], grad_fine.shape[-1]
    N.check(N.lib().dr_mip_downsample_bwd(grad_coarse.data_ptr(), _images(grad_fine), h, w, c,
                                          grad_fine.data_ptr(), N.ptr(out),
                                          0 if out is None else out.shape[-1],
                                          N.stream(grad_fine.device)),
            "dr_mip_downsample_bwd")  # fmt: skip


@timed("edge_neighbours")
def edge_neighbours(tri: Tensor) -> Tensor:
    num_tri = tri.shape[0]
    out = torch.empty((num_tri, 3), dtype=torch.int64, device=tri.device)
    if num_tri == 0:
        return out
    lib = N.lib()
    ws = _scratch(lib.dr_edge_neighbours_workspace_bytes(num_tri), tri.device)
    N.check(lib.dr_edge_neighbours(tri.data_ptr(), num_tri, out.data_ptr(), ws.data_ptr(),
                                   ws.numel(), N.stream(tri.device)), "dr_edge_neighbours")  # fmt: skip
    return out


def edge_opposite(tri: Tensor, neighbours: Tensor) -> Tensor:
    """Vertex opposite each edge in the adjacent triangle (-1 where there is no single one),
    int32 ``[triangles, 3]``: the antialias kernels' form of the adjacency."""
    out = torch.empty((tri.shape[0], 3), dtype=torch.int32, device=tri.device)
    if tri.shape[0]:
        N.check(N.lib().dr_edge_opposite_vertices(tri.data_ptr(), neighbours.data_ptr(),
                                                  tri.shape[0], out.data_ptr(),
                                                  N.stream(tri.device)),
                "dr_edge_opposite_vertices")  # fmt: skip
    return out


def silhouette_edges(pos3: Tensor, tri: Tensor, neighbours: Tensor) -> Tensor:
    opposite = edge_opposite(tri, neighbours)
    out = torch.empty((pos3.shape[0], tri.shape[0], 3), dtype=torch.uint8, device=pos3.device)
    N.check(N.lib().dr_silhouette_edges(pos3.data_ptr(), pos3.shape[0], pos3.shape[1],
                                        tri.data_ptr(), tri.shape[0], opposite.data_ptr(),
                                        out.data_ptr(), N.stream(pos3.device)),
            "dr_silhouette_edges")  # fmt: skip
    return out.bool()


@timed("antialias_fwd")
def antialias_fwd(color, rast, pos3, tri, opposite, record_pairs: bool = False):
    """Antialiased colour, and the pair records for the backward pass when ``record_pairs``."""
    batch, height, width, channels = color.shape
    out = torch.empty_like(color)
    pairs = None
    if record_pairs:
        nbytes = N.lib().dr_antialias_pair_bytes(batch, height, width)
        pairs = torch.empty(nbytes, dtype=torch.uint8, device=color.device)
    N.check(
        N.lib().dr_antialias_fwd(color.data_ptr(), rast.data_ptr(), pos3.data_ptr(), pos3.shape[0],
                                 pos3.shape[1], tri.data_ptr(), tri.shape[0],
                                 opposite.data_ptr(), batch, height, width, channels,
                                 out.data_ptr(), N.ptr(pairs), 0 if pairs is None else pairs.numel(),
                                 N.stream(color.device)),
        "dr_antialias_fwd",
    )  # fmt: skip
    return out, pairs


@timed("antialias_bwd")
def antialias_bwd(color, rast, pos3, tri, opposite, grad_out, boost, pairs=None):
    """Gradients of colour and positions; ``pairs`` from :func:`antialias_fwd` skips the edge
    tests (same result)."""
    batch, height, width, channels = color.shape
    grad_color = torch.empty_like(color)
    grad_pos = zeros_like(pos3)
    N.check(
        N.lib().dr_antialias_bwd(color.data_ptr(), rast.data_ptr(), pos3.data_ptr(), pos3.shape[0],
                                 pos3.shape[1], tri.data_ptr(), tri.shape[0],
                                 opposite.data_ptr(), batch, height, width, channels,
                                 grad_out.data_ptr(), float(boost), N.ptr(pairs),
                                 0 if pairs is None else pairs.numel(), grad_color.data_ptr(),
                                 grad_pos.data_ptr(), N.stream(color.device)),
        "dr_antialias_bwd",
    )  # fmt: skip
    return grad_color, grad_pos


@timed("lambert_fwd")
def lambert_fwd(color: Tensor, normal: Tensor, light: Tensor, ambient: float) -> Tensor:
    """``color * (ambient + max(0, n . l))``; ``normal`` ``[batch, h, w, 3]`` with any uniform
    pixel stride (a channel slice of interpolate's output is read in place)."""
    batch, height, width, channels = color.shape
    normal, stride = pixel_rows(normal)
    out = torch.empty_like(color)
    N.check(
        N.lib().dr_lambert_fwd(color.data_ptr(), normal.data_ptr(), stride, light.data_ptr(),
                               light.shape[0], float(ambient), batch, height, width, channels,
                               out.data_ptr(), N.stream(color.device)),
        "dr_lambert_fwd",
    )  # fmt: skip
    return out


@timed("lambert_bwd")
def lambert_bwd(color, normal, light, ambient, grad_out, need_color: bool, need_normal: bool):
    """Gradients of color and normal (contiguous ``[batch, h, w, 3]``), None where not needed."""
    batch, height, width, channels = color.shape
    normal, stride = pixel_rows(normal)
    grad_color = torch.empty_like(color) if need_color else None
    grad_normal = (torch.empty((batch, height, width, 3), dtype=torch.float32, device=color.device)
                   if need_normal else None)
    N.check(
        N.lib().dr_lambert_bwd(color.data_ptr(), normal.data_ptr(), stride, light.data_ptr(),
                               light.shape[0], float(ambient), batch, height, width, channels,
                               grad_out.data_ptr(), N.ptr(grad_color), N.ptr(grad_normal),
                               N.stream(color.device)),
        "dr_lambert_bwd",
    )  # fmt: skip
    return grad_color, grad_normal


@timed("to_clip_fwd")
def to_clip_fwd(positions: Tensor, matrix: Tensor) -> Tensor:
    """``[batch, V, 4]`` clip positions of ``positions`` ``[V, 3]`` under ``matrix``
    ``[batch, 4, 4]``."""
    clip = torch.empty((matrix.shape[0], positions.shape[0], 4), dtype=torch.float32,
                       device=positions.device)
    N.check(
        N.lib().dr_to_clip_fwd(positions.data_ptr(), positions.shape[0], matrix.data_ptr(),
                               matrix.shape[0], clip.data_ptr(), N.stream(positions.device)),
        "dr_to_clip_fwd",
    )  # fmt: skip
    return clip


@timed("to_clip_bwd")
def to_clip_bwd(grad_clip: Tensor, positions: Tensor, matrix: Tensor, want_positions: bool,
                want_matrix: bool) -> tuple[Tensor | None, Tensor | None]:
    grad_p = torch.empty_like(positions) if want_positions else None
    grad_m = torch.empty_like(matrix) if want_matrix else None
    N.check(
        N.lib().dr_to_clip_bwd(grad_clip.data_ptr(), positions.data_ptr(), positions.shape[0],
                               matrix.data_ptr(), matrix.shape[0], N.ptr(grad_p), N.ptr(grad_m),
                               N.stream(positions.device)),
        "dr_to_clip_bwd",
    )  # fmt: skip
    return grad_p, grad_m


@timed("antialias_fwd")
def antialias_mse_fwd(color, rast, pos3, tri, opposite, target):
    """Antialiased colour, the residual out - target, the pair records and the per-block partial
    sums of the squared residual."""
    batch, height, width, channels = color.shape
    lib = N.lib()
    out = torch.empty_like(color)
    residual = torch.empty_like(color)
    pairs = torch.empty(lib.dr_antialias_pair_bytes(batch, height, width), dtype=torch.uint8,
                        device=color.device)
    partial = torch.zeros(max(1, lib.dr_antialias_loss_partials(batch, height, width)),
                          dtype=torch.float32, device=color.device)
    N.check(
        lib.dr_antialias_mse_fwd(color.data_ptr(), rast.data_ptr(), pos3.data_ptr(), pos3.shape[0],
                                 pos3.shape[1], tri.data_ptr(), tri.shape[0], opposite.data_ptr(),
                                 batch, height, width, channels, target.data_ptr(), out.data_ptr(),
                                 residual.data_ptr(), pairs.data_ptr(), pairs.numel(), partial.data_ptr(),
                                 partial.numel(), N.stream(color.device)),
        "dr_antialias_mse_fwd",
    )  # fmt: skip
    return out, residual, pairs, partial


@timed("antialias_bwd")
def antialias_mse_bwd(color, rast, pos3, tri, opposite, residual, loss_grad, scale, grad_out, boost,
                      pairs):
    """Gradients of colour and positions of ``scale * sum (out - target)^2`` (upstream gradient
    ``loss_grad``, a device scalar) plus ``grad_out`` (the output's own gradient, or None)."""
    batch, height, width, channels = color.shape
    grad_color = torch.empty_like(color)
    grad_pos = zeros_like(pos3)
    N.check(
        N.lib().dr_antialias_mse_bwd(color.data_ptr(), rast.data_ptr(), pos3.data_ptr(),
                                     pos3.shape[0], pos3.shape[1], tri.data_ptr(), tri.shape[0],
                                     opposite.data_ptr(), batch, height, width, channels,
                                     residual.data_ptr(), loss_grad.data_ptr(), float(scale),
                                     N.ptr(grad_out), float(boost), pairs.data_ptr(),
                                     pairs.numel(), grad_color.data_ptr(), grad_pos.data_ptr(),
                                     N.stream(color.device)),
        "dr_antialias_mse_bwd",
    )  # fmt: skip
    return grad_color, grad_pos


def capture_overflowed(device: torch.device) -> bool:
    """Whether a captured visibility pass on ``device`` exceeded its capacities since the last
    call (synchronizes); if so, the capacities for later captures are doubled."""
    word = _overflow.get(device)
    if word is None or int(word.item()) == 0:
        return False
    word.zero_()
    for key, (cap, pair_cap) in list(_graph_capacity.items()):
        if key[0] == device:
            _graph_capacity[key] = (2 * cap, 2 * pair_cap)
    return True
