"""Autograd functions over the CUDA kernels. Inputs arrive validated (see ``ops.py``).

Each backward runs hand-written kernels with no second-order terms, so a backward pass asked to
build a graph (``create_graph=True``) raises, like the reference's first-order guard
(diffrast backends/_autograd.py:11-35).
"""

from __future__ import annotations

import functools

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


class Rasterize(torch.autograd.Function):
    """Visibility, then rast / rast_db; gradients reach pos through the barycentric resolve."""

    @staticmethod
    def forward(ctx, pos: Tensor, tri: Tensor, height: int, width: int, grad_db: bool,
                prev_keys: Tensor | None, ranges: K.RangeTable | None):
        keys = K.raster_keys(pos, tri, height, width, prev_keys, ranges)
        rast, rast_db = K.resolve_fwd(pos, tri, keys)
        # Unused outputs (keys always, rast_db often) get no zero-filled gradient.
        ctx.set_materialize_grads(False)
        ctx.save_for_backward(_saveable(pos), _saveable(tri), keys)
        ctx.grad_db = grad_db
        ctx.mark_non_differentiable(keys)
        if not grad_db:
            ctx.mark_non_differentiable(rast_db)
        return rast, rast_db, keys

    @staticmethod
    @first_order("rasterize")
    def backward(ctx, grad_rast, grad_db, _grad_keys):
        pos, tri, keys = ctx.saved_tensors
        if grad_rast is None:
            grad_rast = torch.zeros((*keys.shape, 4), dtype=pos.dtype, device=pos.device)
        use_db = ctx.grad_db and grad_db is not None
        grad_pos = K.resolve_bwd(pos, tri, keys, K.aligned(grad_rast),
                                 K.aligned(grad_db) if use_db else None)
        return grad_pos, None, None, None, None, None, None


class Interpolate(torch.autograd.Function):
    @staticmethod
    def forward(ctx, attr: Tensor, rast: Tensor, rast_db: Tensor | None, tri: Tensor,
                diff: Tensor | None):
        attr3 = (attr if attr.ndim == 3 else attr[None]).contiguous()
        channels = attr3.shape[2]
        # Rows padded to 16 bytes for the forward kernel's vector loads.
        attr_rows, _ = K.padded_rows(attr3)
        out, out_da = K.interpolate_fwd(attr_rows, rast, rast_db, tri, diff, channels)
        ctx.set_materialize_grads(False)
        ctx.save_for_backward(*(_saveable(t) for t in (attr3, rast, rast_db, tri, diff)))
        ctx.attr_shape = attr.shape
        ctx.channels = channels
        ctx.has_da = diff is not None
        ctx.rast_db_given = rast_db is not None
        if diff is None:
            ctx.mark_non_differentiable(out_da)
        return out, out_da

    @staticmethod
    @first_order("interpolate")
    def backward(ctx, grad_out, grad_out_da):
        attr3, rast, rast_db, tri, diff = ctx.saved_tensors
        if grad_out is None:
            grad_out = torch.zeros((*rast.shape[:3], ctx.channels), device=rast.device)
        use_da = ctx.has_da and grad_out_da is not None
        need_attr = ctx.needs_input_grad[0]
        grad_attr, grad_rast, grad_db = K.interpolate_bwd(
            attr3, rast, rast_db, tri, diff if use_da else None, grad_out.contiguous(),
            grad_out_da.contiguous() if use_da else None, need_attr,
        )
        if not ctx.rast_db_given:
            grad_db = None
        if grad_attr is not None:
            grad_attr = grad_attr.view(ctx.attr_shape)
        return grad_attr, grad_rast, grad_db, None, None


class MipChain(torch.autograd.Function):
    """Levels 1.. of a texture by repeated area-weighted halving; backward is the adjoint chain."""

    @staticmethod
    def forward(ctx, tex: Tensor, count: int):
        levels = []
        level = tex
        for _ in range(count):
            level = K.mip_down(level)
            levels.append(level)
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
    ``da_spec`` = (first channel, count)), such as interpolate's outputs: their gradients are then
    written straight into gradients of the wider tensors instead of being copied there by the
    slices' own backward."""

    @staticmethod
    def forward(ctx, uv_src, da_src, bias, mode: int, boundary: int, uv_spec, da_spec, *levels):
        levels = [lv.contiguous() for lv in levels]
        out = K.texture_fwd(list(levels), _take(uv_src, uv_spec), _take(da_src, da_spec), bias,
                            mode, boundary)
        ctx.save_for_backward(*(_saveable(t) for t in (uv_src, da_src, bias, *levels)))
        ctx.settings = (mode, boundary, da_src is not None, bias is not None, len(levels))
        ctx.specs = (uv_spec, da_spec)
        return out

    @staticmethod
    @first_order("texture")
    def backward(ctx, grad_out):
        mode, boundary, has_da, has_bias, count = ctx.settings
        uv_spec, da_spec = ctx.specs
        saved = ctx.saved_tensors
        uv_src, da_src, bias, levels = saved[0], saved[1], saved[2], list(saved[3:])
        need = ctx.needs_input_grad
        want_uv = need[0] and mode > 0
        want_da = need[1] and has_da and mode == 3
        want_bias = need[2] and has_bias and mode == 3
        g_uv_src, uv_first = _slice_gradient(uv_src, uv_spec, want_uv)
        g_da_src, da_first = _slice_gradient(da_src, da_spec, want_da)
        grads, g_uv, g_da, g_bias = K.texture_bwd(levels, _take(uv_src, uv_spec),
                                                  _take(da_src, da_spec), bias, mode, boundary,
                                                  grad_out.contiguous(), want_uv, want_da,
                                                  want_bias, grad_uv=g_uv_src, grad_da=g_da_src,
                                                  uv_first=uv_first, da_first=da_first)
        g_uv = g_uv_src if uv_spec is not None else g_uv
        g_da = g_da_src if da_spec is not None else g_da
        level_grads = [g if need[7 + i] else None for i, g in enumerate(grads)]
        return (g_uv, g_da, g_bias, None, None, None, None, *level_grads)


class TextureChain(torch.autograd.Function):
    """Mipmapped lookup with the mip chain of ``tex`` built inside the function.

    The levels never enter the autograd graph: the backward pass accumulates the gradients of all
    levels (in 4-channel buffers when the texture has 3 channels), pushes them down the chain with
    the adjoint kernel in place, and returns only the base level's gradient.
    """

    @staticmethod
    def forward(ctx, uv_src, da_src, bias, mode: int, boundary: int, count: int, tex: Tensor,
                uv_spec=None, da_spec=None):
        tex = tex.contiguous()
        levels = [tex]
        for _ in range(count):
            levels.append(K.mip_down(levels[-1]))
        out = K.texture_fwd(levels, _take(uv_src, uv_spec), _take(da_src, da_spec), bias, mode,
                            boundary)
        ctx.save_for_backward(*(_saveable(t) for t in (uv_src, da_src, bias, tex)))
        ctx.levels = levels[1:]
        ctx.settings = (mode, boundary)
        ctx.specs = (uv_spec, da_spec)
        return out

    @staticmethod
    @first_order("texture")
    def backward(ctx, grad_out):
        mode, boundary = ctx.settings
        uv_spec, da_spec = ctx.specs
        uv_src, da_src, bias, tex = ctx.saved_tensors
        levels = [tex, *ctx.levels]
        need = ctx.needs_input_grad
        want_uv = need[0] and mode > 0
        want_da = need[1] and da_src is not None and mode == 3
        want_bias = need[2] and bias is not None and mode == 3
        g_uv_src, uv_first = _slice_gradient(uv_src, uv_spec, want_uv)
        g_da_src, da_first = _slice_gradient(da_src, da_spec, want_da)
        grads, g_uv, g_da, g_bias = K.texture_bwd(levels, _take(uv_src, uv_spec),
                                                  _take(da_src, da_spec), bias, mode, boundary,
                                                  grad_out.contiguous(), want_uv, want_da,
                                                  want_bias, keep_padded=True, grad_uv=g_uv_src,
                                                  grad_da=g_da_src, uv_first=uv_first,
                                                  da_first=da_first)
        g_uv = g_uv_src if uv_spec is not None else g_uv
        g_da = g_da_src if da_spec is not None else g_da
        grad_tex = None
        if need[6]:
            padded = grads[0].shape[-1] != tex.shape[-1]
            for level in range(len(grads) - 2, -1, -1):
                # The last step writes the base gradient without the padding channel.
                last = level == 0 and padded
                out = torch.empty(tex.shape, dtype=torch.float32, device=tex.device) if last else None
                K.mip_down_bwd(grads[level + 1], grads[level], out)
                if last:
                    grads[0] = out
            grad_tex = grads[0]
            if grad_tex.shape[-1] != tex.shape[-1]:
                grad_tex = grad_tex[..., : tex.shape[-1]].contiguous()
        return g_uv, g_da, g_bias, None, None, None, grad_tex, None, None


class Antialias(torch.autograd.Function):
    @staticmethod
    def forward(ctx, color: Tensor, rast: Tensor, pos: Tensor, tri: Tensor, opposite: Tensor,
                boost: float):
        pos3 = pos if pos.ndim == 3 else pos[None]
        # The pair records (about 25 bytes per pixel) spare the backward pass the edge tests.
        out, pairs = K.antialias_fwd(color, rast, pos3, tri, opposite,
                                     record_pairs=any(ctx.needs_input_grad[:3]))
        saved = (color, rast, pos3, tri, opposite, pairs)
        ctx.save_for_backward(*(_saveable(t) for t in saved))
        ctx.boost = boost
        ctx.pos_shape = pos.shape
        return out

    @staticmethod
    @first_order("antialias")
    def backward(ctx, grad_out):
        color, rast, pos3, tri, opposite, pairs = ctx.saved_tensors
        grad_color, grad_pos = K.antialias_bwd(color, rast, pos3, tri, opposite,
                                               grad_out.contiguous(), ctx.boost, pairs)
        return grad_color, None, grad_pos.view(ctx.pos_shape), None, None, None


class AntialiasMSE(torch.autograd.Function):
    """Antialias with the squared-error loss ``scale * sum (out - target)^2`` fused into its
    passes; returns ``(out, loss)``."""

    @staticmethod
    def forward(ctx, color: Tensor, rast: Tensor, pos: Tensor, tri: Tensor, opposite: Tensor,
                target: Tensor, scale: float, boost: float):
        pos3 = pos if pos.ndim == 3 else pos[None]
        out, residual, pairs, partial = K.antialias_mse_fwd(color, rast, pos3, tri, opposite, target)
        loss = partial.sum() * scale
        ctx.set_materialize_grads(False)
        saved = (color, rast, pos3, tri, opposite, pairs, residual)
        ctx.save_for_backward(*(_saveable(t) for t in saved))
        ctx.scale, ctx.boost, ctx.pos_shape = scale, boost, pos.shape
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
        return grad_color, None, grad_pos.view(ctx.pos_shape), None, None, None, None, None


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
