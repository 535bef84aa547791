"""CPU restatement of diffrast's reference backend, restricted to the render path.

TEST INFRASTRUCTURE ONLY. This module is the checker for the CUDA kernels of ``diffrast_b200``
and the timed CPU baseline of ``bench.py``; the product never imports it. Its parity with the
reference is pinned by the golden fixtures under ``tests/golden/`` (made by running the reference
package itself, see ``tests/golden/make_golden.py``).

Everything runs in float32 on the CPU with PyTorch, and gradients come from autograd, as in the
reference backend (``src/diffrast/backends/reference.py:1-13``). The visibility arithmetic
(``coverage``) performs the reference's float32 operations one for one and in the same order
(``reference.py:293-365``): that is what makes triangle ids comparable bit for bit. Everything else
follows the reference's formulas, organised in this module's own way (flat per-pixel lists, a
separable weight matrix for the mip chain, an explicit per-level loop for mipmapped lookups).

Paths cited as ``reference.py``, ``_cube.py``, ``ops.py`` are files of the reference project under
``src/diffrast/`` (``backends/reference.py``, ``backends/_cube.py``, ``ops.py``).
"""

from __future__ import annotations

import math
from collections.abc import Sequence

import numpy as np
import torch
from torch import Tensor

__all__ = [
    "AREA_TOLERANCE",
    "AXIS_TIE",
    "EDGE_TIE",
    "EMPTY_KEY",
    "antialias",
    "coverage",
    "cube_fold",
    "cube_project",
    "edge_neighbours",
    "interpolate",
    "keys_from_state",
    "mip_chain",
    "pixel_centres",
    "rasterize",
    "rasterize_layer",
    "resolve",
    "resolve_at_pixels",
    "silhouette_edges",
    "texture",
    "visible_at_pixels",
    "visible_triangles",
]

# Numeric contracts of the reference (reference.py:23-35, :402; _cube.py:36).
AREA_TOLERANCE = 2
AXIS_TIE = 1 + 1e-4
EDGE_TIE = 4
FOOTPRINT_LIMIT = 1e18
DERIVATIVE_LIMIT = 1e18
EPS32 = float(torch.finfo(torch.float32).eps)
TINY32 = float(torch.finfo(torch.float32).tiny)
# Pixels x triangles evaluated at once by the brute-force visibility pass; any value gives the
# same result, it only bounds memory.
_BLOCK_ELEMENTS = 1 << 21
EMPTY_KEY = (1 << 63) - 1


# --------------------------------------------------------------------------------------------
# Rasterization
# --------------------------------------------------------------------------------------------


def pixel_centres(height: int, width: int) -> tuple[Tensor, Tensor]:
    """NDC x of every column and y of every row: ``(2 i + 1) / size - 1`` in float32.

    Follows ``reference.py:268-271``: the division is IEEE float32 division.
    """
    cols = torch.arange(width, dtype=torch.float32)
    rows = torch.arange(height, dtype=torch.float32)
    return (cols * 2 + 1) / width - 1, (rows * 2 + 1) / height - 1


def _edge_terms(x, y, w, px, py):
    """``a_k = x_k - px w_k``, ``c_k = y_k - py w_k`` and ``e_k = a_i c_j - a_j c_i``.

    ``i = k + 1`` and ``j = k + 2`` modulo 3, so ``e_k`` is the edge opposite vertex ``k``
    (``reference.py:274-278``, ``:303-307``). ``x``, ``y``, ``w`` are lists of three tensors.
    """
    a = [x[k] - px * w[k] for k in range(3)]
    c = [y[k] - py * w[k] for k in range(3)]
    e = [a[(k + 1) % 3] * c[(k + 2) % 3] - a[(k + 2) % 3] * c[(k + 1) % 3] for k in range(3)]
    return a, c, e


def coverage(x, y, z, w, px, py) -> tuple[Tensor, Tensor]:
    """Inside test and depth ``z / w`` of triangles at pixel centres.

    ``x, y, z, w`` are lists of the three vertices' coordinates, broadcastable against ``px`` and
    ``py``. The float32 operations and their order are those of ``reference.py:293-365``:
    homogeneous edge functions, the top-left tie rule on exact zeros, the area tolerance of two
    epsilons relative to the magnitude of the terms, the sign of the interpolated ``w``, the depth
    range ``[-1, 1]`` and finiteness of every coordinate.
    """
    a, c, e = _edge_terms(x, y, w, px, py)
    s = e[0] + e[1] + e[2]
    ew = e[0] * w[0] + e[1] * w[1] + e[2] * w[2]
    depth = (e[0] * z[0] + e[1] * z[1] + e[2] * z[2]) / ew
    positive = s > 0

    inside = None
    for k in range(3):
        i, j = (k + 1) % 3, (k + 2) % 3
        # Direction of the screen-space gradient of e_k decides a pixel exactly on the edge
        # (reference.py:338-365).
        gx = c[i] * w[j] - c[j] * w[i]
        gy = a[j] * w[i] - a[i] * w[j]
        q = torch.where(e[k] == 0, torch.where(gx == 0, gy, gx), e[k])
        side = torch.where(positive, q > 0, q < 0)
        inside = side if inside is None else inside & side

    reach_x = torch.maximum(
        torch.maximum(x[0].abs() + w[0].abs(), x[1].abs() + w[1].abs()), x[2].abs() + w[2].abs()
    )
    reach_y = torch.maximum(
        torch.maximum(y[0].abs() + w[0].abs(), y[1].abs() + w[1].abs()), y[2].abs() + w[2].abs()
    )
    span_x = a[0].abs() + a[1].abs() + a[2].abs()
    span_y = c[0].abs() + c[1].abs() + c[2].abs()
    tolerance = AREA_TOLERANCE * EPS32
    inside = inside & (s.abs() > (reach_x * span_y + span_x * (reach_y + span_y)) * tolerance)
    inside = inside & torch.where(positive, ew > 0, ew < 0)
    inside = inside & (depth >= -1) & (depth <= 1)
    finite = None
    for comp in (x, y, z, w):
        for k in range(3):
            f = torch.isfinite(comp[k])
            finite = f if finite is None else finite & f
    return inside & finite, depth


def visible_triangles(
    pos: Tensor,
    tri: Tensor,
    height: int,
    width: int,
    previous: tuple[Tensor, Tensor] | None = None,
) -> tuple[Tensor, Tensor]:
    """Brute-force nearest covering triangle per pixel (``reference.py:368-397``).

    Returns ``(depth, tri_id)`` of shape ``[batch, height, width]``: float32 depth (``inf`` where
    empty) and int64 index (``-1`` where empty). Equal depths go to the lower index. With
    ``previous`` (the state of an earlier layer) only triangles ordered after it by
    ``(depth, index)`` count.
    """
    pos = pos.detach().float()
    tri = tri.long()
    batch, num_tri = pos.shape[0], tri.shape[0]
    px, py = pixel_centres(height, width)
    px, py = px.view(1, 1, 1, width), py.view(1, 1, height, 1)
    best_depth = torch.full((batch, height, width), math.inf)
    best_id = torch.full((batch, height, width), -1, dtype=torch.long)
    block = max(1, _BLOCK_ELEMENTS // max(1, batch * height * width))
    if previous is not None:
        prev_depth, prev_id = previous[0][:, None], previous[1][:, None]
    for start in range(0, num_tri, block):
        idx = tri[start : start + block]
        v = pos[:, idx][:, :, :, None, None, :]  # [B, n, 3, 1, 1, 4]
        coords = [[v[:, :, k, ..., comp] for k in range(3)] for comp in range(4)]
        inside, depth = coverage(*coords, px, py)
        ids = torch.arange(start, start + idx.shape[0]).view(1, -1, 1, 1)
        if previous is not None:
            later = (depth > prev_depth) | ((depth == prev_depth) & (ids > prev_id))
            inside = inside & later
        depth = torch.where(inside, depth, torch.full_like(depth, math.inf))
        near = depth.amin(1)
        first = torch.where(inside & (depth == near[:, None]), ids, num_tri).amin(1)
        closer = near < best_depth
        best_depth = torch.where(closer, near, best_depth)
        best_id = torch.where(closer, first, best_id)
    return best_depth, best_id


def visible_at_pixels(
    pos: Tensor, tri: Tensor, height: int, width: int, rows: Tensor, cols: Tensor,
    margin_px: float = 2.0,
) -> tuple[Tensor, Tensor]:
    """``visible_triangles`` of one view (``pos [V, 4]``) at listed pixels only.

    Returns ``(depth, tri_id)`` of shape ``[N]`` for the pixels ``(rows[n], cols[n])`` of an
    ``height x width`` image. Coverage is the exact ``coverage`` test, run for each pixel on every
    triangle that can reach it: those with a vertex at ``w <= 0`` or non-finite, and those whose
    projected bounding box, grown by ``margin_px`` pixels, contains the pixel centre. A triangle
    with all ``w > 0`` covers only points of its projected triangle, which lies inside that box
    (the margin is far above the rounding of the projection), so the result equals
    ``visible_triangles`` at those pixels; it exists so that images of a million triangles can be
    checked at a few thousand pixels.
    """
    pos = pos.detach().float()
    tri = tri.long()
    num_tri = tri.shape[0]
    px_all, py_all = pixel_centres(height, width)
    px, py = px_all[cols.long()], py_all[rows.long()]
    v = pos[tri]  # [T, 3, 4]
    w = v[..., 3]
    finite = torch.isfinite(v).all(-1).all(-1)
    front = (w > 0).all(-1) & finite
    safe_w = torch.where(front[:, None], w, torch.ones_like(w))
    sx, sy = v[..., 0] / safe_w, v[..., 1] / safe_w
    mx, my = 2.0 * margin_px / width, 2.0 * margin_px / height
    x0, x1 = sx.amin(-1) - mx, sx.amax(-1) + mx
    y0, y1 = sy.amin(-1) - my, sy.amax(-1) + my
    always = (~front).nonzero().flatten()
    depth_out = torch.full((px.shape[0],), math.inf)
    id_out = torch.full((px.shape[0],), -1, dtype=torch.long)
    # Pixels are handled in groups of one 8 x 8 cell: the candidates of a cell are the triangles
    # whose grown box meets the cell's pixel-centre rectangle.
    cell = (rows.long() // 8) * ((width + 7) // 8) + cols.long() // 8
    for c in cell.unique().tolist():
        members = (cell == c).nonzero().flatten()
        cx, cy = px[members], py[members]
        reach = front & (x0 <= cx.max()) & (x1 >= cx.min()) & (y0 <= cy.max()) & (y1 >= cy.min())
        cand = torch.cat([reach.nonzero().flatten(), always]).unique()
        if cand.numel() == 0:
            continue
        vc = v[cand][:, :, None, :]  # [n, 3, 1, 4] against [members]
        coords = [[vc[:, k, :, comp] for k in range(3)] for comp in range(4)]
        inside, depth = coverage(*coords, cx[None], cy[None])  # [n, members]
        depth = torch.where(inside, depth, torch.full_like(depth, math.inf))
        near = depth.amin(0)
        ids = cand[:, None].expand_as(depth)
        first = torch.where(inside & (depth == near[None]), ids, torch.full_like(ids, num_tri)).amin(0)
        hit = near < math.inf
        depth_out[members[hit]] = near[hit]
        id_out[members[hit]] = first[hit]
    return depth_out, id_out


def keys_from_state(depth: Tensor, tri_id: Tensor) -> Tensor:
    """Packed 64-bit visibility keys ``(ordered depth bits << 32) | id`` from a layer's state.

    The ordered integer of a float32 keeps its order (``bits`` if non-negative, else
    ``bits ^ 0x7FFFFFFF``) with -0 mapped to 0; empty pixels get ``EMPTY_KEY``. This is the state
    format of the CUDA rasterizer, so tests can compare states directly.
    """
    bits = depth.contiguous().view(torch.int32).long()
    ordered = torch.where(bits >= 0, bits, bits ^ 0x7FFFFFFF)
    ordered = torch.where(depth == 0, torch.zeros_like(ordered), ordered)
    key = (ordered << 32) | tri_id.clamp(min=0)
    return torch.where(tri_id >= 0, key, torch.full_like(key, EMPTY_KEY))


def resolve(pos: Tensor, tri: Tensor, tri_id: Tensor, grad_db: bool = True) -> tuple[Tensor, Tensor]:
    """``rast`` and ``rast_db`` of the visible triangles, differentiable in ``pos``.

    Formulas of ``reference.py:69-114``: ``b = e / sum(e)``, depth ``sum(b z) / sum(b w)``,
    ``de/dpx = c x w``, ``de/dpy = w x a``, ``db = (de - b sum(de)) / sum(e)``, scaled by the NDC
    size of a pixel, ``2 / width`` and ``2 / height``.
    """
    batch, height, width = tri_id.shape
    px, py = pixel_centres(height, width)
    bi, ri, ci = (tri_id >= 0).nonzero(as_tuple=True)
    seen = tri_id[bi, ri, ci]
    v = pos[bi[:, None], tri.long()[seen]]  # [N, 3, 4]
    values, derivs = _resolve_points(v, px[ci].to(pos.dtype), py[ri].to(pos.dtype), seen, height,
                                     width, grad_db)
    rast = pos.new_zeros(batch, height, width, 4).index_put((bi, ri, ci), values)
    rast_db = pos.new_zeros(batch, height, width, 4).index_put((bi, ri, ci), derivs)
    return rast, rast_db


def resolve_at_pixels(pos: Tensor, tri: Tensor, height: int, width: int, rows: Tensor,
                      cols: Tensor, tri_id: Tensor) -> tuple[Tensor, Tensor]:
    """``rast`` and ``rast_db`` ``[N, 4]`` of one view (``pos [V, 4]``) at listed pixels whose
    visible triangles are ``tri_id [N]`` (-1: empty, zeros), in ``pos``'s dtype (float64 gives the
    reference values the CUDA results are compared with)."""
    px, py = pixel_centres(height, width)
    hit = (tri_id >= 0).nonzero().flatten()
    seen = tri_id[hit]
    v = pos[tri.long()[seen]]  # [N, 3, 4]
    values, derivs = _resolve_points(v, px[cols[hit].long()].to(pos.dtype),
                                     py[rows[hit].long()].to(pos.dtype), seen, height, width, True)
    rast = pos.new_zeros(tri_id.shape[0], 4)
    rast_db = pos.new_zeros(tri_id.shape[0], 4)
    rast[hit], rast_db[hit] = values, derivs
    return rast, rast_db


def _resolve_points(v, pxn, pyn, seen, height, width, grad_db):
    """Barycentrics, depth, id + 1 and their screen derivatives of triangles ``v [N, 3, 4]`` at
    the pixel centres ``(pxn, pyn)``."""
    x, y, z, w = ([v[:, k, comp] for k in range(3)] for comp in range(4))
    a, c, e = _edge_terms(x, y, w, pxn, pyn)
    area = e[0] + e[1] + e[2]
    b = [ek / area for ek in e]
    depth = (b[0] * z[0] + b[1] * z[1] + b[2] * z[2]) / (b[0] * w[0] + b[1] * w[1] + b[2] * w[2])
    dedx = [w[(k + 2) % 3] * c[(k + 1) % 3] - w[(k + 1) % 3] * c[(k + 2) % 3] for k in range(3)]
    dedy = [a[(k + 2) % 3] * w[(k + 1) % 3] - a[(k + 1) % 3] * w[(k + 2) % 3] for k in range(3)]
    sx, sy = dedx[0] + dedx[1] + dedx[2], dedy[0] + dedy[1] + dedy[2]
    dbdx = [(dedx[k] - b[k] * sx) / area for k in range(2)]
    dbdy = [(dedy[k] - b[k] * sy) / area for k in range(2)]
    if not grad_db:
        dbdx = [t.detach() for t in dbdx]
        dbdy = [t.detach() for t in dbdy]
    values = torch.stack([b[0], b[1], depth, (seen + 1).to(v.dtype)], -1)
    derivs = torch.stack(
        [dbdx[0] * (2 / width), dbdy[0] * (2 / height), dbdx[1] * (2 / width), dbdy[1] * (2 / height)],
        -1,
    )
    return values, derivs


def rasterize_layer(
    pos: Tensor,
    tri: Tensor,
    resolution: tuple[int, int],
    grad_db: bool = True,
    previous: tuple[Tensor, Tensor] | None = None,
) -> tuple[Tensor, Tensor, tuple[Tensor, Tensor]]:
    """One depth layer behind ``previous``: ``(rast, rast_db, state)`` (``reference.py:45-66``)."""
    height, width = resolution
    if tri.shape[0] == 0 or pos.shape[0] == 0:
        empty = pos.new_zeros(pos.shape[0], height, width, 4)
        none = torch.full((pos.shape[0], height, width), -1, dtype=torch.long)
        return empty, empty.clone(), (torch.full(none.shape, math.inf), none)
    with torch.no_grad():
        depth, ids = visible_triangles(pos, tri, height, width, previous)
    rast, rast_db = resolve(pos, tri, ids, grad_db)
    return rast, rast_db, (depth, ids)


def rasterize(pos: Tensor, tri: Tensor, resolution, grad_db: bool = True) -> tuple[Tensor, Tensor]:
    """Instanced-mode rasterization: ``(rast, rast_db)``."""
    rast, rast_db, _ = rasterize_layer(pos, tri, resolution, grad_db, None)
    return rast, rast_db


# --------------------------------------------------------------------------------------------
# Interpolation
# --------------------------------------------------------------------------------------------


def interpolate(
    attr: Tensor, rast: Tensor, tri: Tensor, rast_db: Tensor | None = None, diff: Sequence[int] = ()
) -> tuple[Tensor, Tensor]:
    """Barycentric interpolation and its screen-space derivatives (``reference.py:117-146``).

    ``out = u a0 + v a1 + (1 - u - v) a2``; for each channel in ``diff``,
    ``(du/dx (a0 - a2) + dv/dx (a1 - a2), du/dy (a0 - a2) + dv/dy (a1 - a2))``. Ids past the end of
    ``tri`` count as background.
    """
    diff = list(diff)
    batch, height, width, _ = rast.shape
    channels = attr.shape[-1]
    out = attr.new_zeros(batch, height, width, channels)
    out_da = attr.new_zeros(batch, height, width, 2 * len(diff))
    if tri.shape[0] == 0:
        return out, out_da
    tri_id = rast[..., 3].detach().round().long() - 1
    bi, ri, ci = ((tri_id >= 0) & (tri_id < tri.shape[0])).nonzero(as_tuple=True)
    table = (attr if attr.ndim == 3 else attr[None]).expand(batch, -1, -1)
    corners = table[bi[:, None], tri.long()[tri_id[bi, ri, ci]]]  # [N, 3, C]
    a0, a1, a2 = corners[:, 0], corners[:, 1], corners[:, 2]
    u, v = rast[bi, ri, ci, 0:1], rast[bi, ri, ci, 1:2]
    out = out.index_put((bi, ri, ci), u * a0 + v * a1 + (1 - u - v) * a2)
    if not diff:
        return out, out_da
    d0, d1 = (a0 - a2)[:, diff], (a1 - a2)[:, diff]
    db = rast_db[bi, ri, ci]
    ddx = db[:, 0:1] * d0 + db[:, 2:3] * d1
    ddy = db[:, 1:2] * d0 + db[:, 3:4] * d1
    out_da = out_da.index_put((bi, ri, ci), torch.stack([ddx, ddy], -1).flatten(-2))
    return out, out_da


# --------------------------------------------------------------------------------------------
# Texture
# --------------------------------------------------------------------------------------------


def _halving_weights(n: int) -> Tensor:
    """``[ceil(n / 2), n]`` area weights of one mip step along a dimension of ``n`` texels.

    Bin ``j`` of the coarse level covers ``[j n, (j + 1) n]`` and texel ``i`` covers
    ``[i m, (i + 1) m]`` in units of ``1 / (n m)``, ``m = ceil(n / 2)``; the weight is their
    overlap divided by ``n`` (``reference.py:449-488``; for even ``n`` this is the pair mean).
    """
    m = (n + 1) // 2
    j = torch.arange(m)[:, None]
    i = torch.arange(n)[None, :]
    overlap = torch.minimum((j + 1) * n, (i + 1) * m) - torch.maximum(j * n, i * m)
    return overlap.clamp(min=0).float() / n


def _halve_dim(image: Tensor, dim: int) -> Tensor:
    """One mip step along ``dim``: each coarse texel is a weighted sum of at most three taps.

    The taps and weights are the nonzero entries of :func:`_halving_weights` (gathered, so large
    textures cost O(texels)).
    """
    n = image.shape[dim]
    if n == 1:
        return image
    weights = _halving_weights(n)
    m = weights.shape[0]
    first = torch.arange(m) * n // m
    out = 0
    for tap in range(3):
        idx = (first + tap).clamp(max=n - 1)
        wt = weights[torch.arange(m), idx] * (first + tap < n)
        shape = [1] * image.ndim
        shape[dim] = m
        out = out + wt.view(shape) * image.index_select(dim, idx)
    return out


def _downsample(level: Tensor) -> Tensor:
    """Next mip level of ``[batch, h, w, C]`` as a separable weighted sum."""
    return _halve_dim(_halve_dim(level, 1), 2)


def mip_chain(tex: Tensor, max_mip_level: int | None = None) -> list[Tensor]:
    """Base level and every halving until both sizes are 1 (``reference.py:433-446``).

    A cube map ``[B, 6, s, s, C]`` is filtered face by face.
    """
    cube = tex.ndim == 5
    levels = [tex.flatten(0, 1) if cube else tex]
    while max(levels[-1].shape[1:3]) > 1 and (max_mip_level is None or len(levels) <= max_mip_level):
        levels.append(_downsample(levels[-1]))
    if cube:
        levels = [tex, *(lv.unflatten(0, tex.shape[:2]) for lv in levels[1:])]
    return levels


def _level_of_detail(uv_da: Tensor, height: int, width: int) -> Tensor:
    """``0.5 log2`` of the longer squared footprint axis in texels (``reference.py:491-501``)."""
    lim = FOOTPRINT_LIMIT
    dux, duy, dvx, dvy = uv_da.unbind(-1)
    len_x = (dux * width).clamp(-lim, lim) ** 2 + (dvx * height).clamp(-lim, lim) ** 2
    len_y = (duy * width).clamp(-lim, lim) ** 2 + (dvy * height).clamp(-lim, lim) ** 2
    return 0.5 * torch.log2(torch.maximum(len_x, len_y).clamp_min(1e-30))


_MAJOR = ((1, 0, 0), (-1, 0, 0), (0, 1, 0), (0, -1, 0), (0, 0, 1), (0, 0, -1))
_S_AXIS = ((0, 0, -1), (0, 0, 1), (1, 0, 0), (1, 0, 0), (1, 0, 0), (-1, 0, 0))
_T_AXIS = ((0, -1, 0), (0, -1, 0), (0, 0, 1), (0, 0, -1), (0, -1, 0), (0, -1, 0))


def cube_project(dirs: Tensor, dirs_da: Tensor | None = None):
    """Face, face coordinates ``st``, their derivatives and validity of directions.

    OpenGL face table and tie order x > y > z (``_cube.py:1-102``). Invalid directions (non-finite,
    or largest magnitude below the smallest normal float) get a placeholder ``(0, 0, 1)``.
    Derivatives are divided by the length (largest magnitude), saturated at ``1e18`` and chained by
    the quotient rule; a NaN derivative of a valid direction gives NaN ``st_da``.
    """
    major_t, s_t, t_t = (torch.tensor(t, dtype=dirs.dtype) for t in (_MAJOR, _S_AXIS, _T_AXIS))
    valid = torch.isfinite(dirs).all(-1) & (dirs.detach().abs().amax(-1) >= TINY32)
    dirs = torch.where(valid[..., None], dirs, dirs.new_tensor((0.0, 0.0, 1.0)))
    ax, ay, az = dirs.detach().abs().unbind(-1)
    x_major = (ax >= ay) & (ax >= az)
    y_major = ~x_major & (ay >= az)
    axis = 2 - 2 * x_major.long() - y_major.long()
    negative = dirs.detach().gather(-1, axis[..., None]).squeeze(-1) < 0
    face = 2 * axis + negative.long()
    length = dirs.detach().abs().amax(-1, keepdim=True)
    unit = dirs / length
    major, s_ax, t_ax = major_t[face], s_t[face], t_t[face]
    ma = (unit * major).sum(-1, keepdim=True)
    ratio = torch.stack([(unit * s_ax).sum(-1), (unit * t_ax).sum(-1)], -1) / ma
    st = 0.5 * (ratio + 1)
    if dirs_da is None:
        return face, st, None, valid
    undefined = valid & dirs_da.isnan().any(-1)
    da = torch.where((valid & ~undefined)[..., None], dirs_da, 0) / length
    da = da.clamp(-DERIVATIVE_LIMIT, DERIVATIVE_LIMIT).unflatten(-1, (3, 2))
    d_ma = (da * major[..., None]).sum(-2)
    d_sc = (da * s_ax[..., None]).sum(-2)
    d_tc = (da * t_ax[..., None]).sum(-2)
    ds = 0.5 * (d_sc - ratio[..., :1] * d_ma) / ma
    dt = 0.5 * (d_tc - ratio[..., 1:] * d_ma) / ma
    st_da = torch.where(undefined[..., None], torch.nan, torch.cat([ds, dt], -1))
    return face, st, st_da, valid


def cube_fold(face: Tensor, row: Tensor, col: Tensor, size: Tensor):
    """Move texel coordinates one step outside a face onto the neighbouring face.

    Integer geometry in half-texel units (``_cube.py:105-143``): the texel centre is placed on the
    cube surface, pulled one half-texel inwards along the old major axis when it sticks out, and
    re-projected. Coordinates outside two edges (beyond a corner) do not exist.
    """
    major_t, s_t, t_t = (torch.tensor(t, dtype=torch.long) for t in (_MAJOR, _S_AXIS, _T_AXIS))
    major, s_ax, t_ax = major_t[face], s_t[face], t_t[face]
    over_col = (col < 0) | (col >= size)
    over_row = (row < 0) | (row >= size)
    ext = size[..., None]
    point = (ext * major + (2 * col + 1 - size)[..., None] * s_ax + (2 * row + 1 - size)[..., None] * t_ax)
    point = torch.maximum(torch.minimum(point, ext), -ext)
    point = point - (over_col | over_row)[..., None] * major
    axis = point.abs().argmax(-1)
    negative = point.gather(-1, axis[..., None]).squeeze(-1) < 0
    new_face = 2 * axis + negative.long()
    s2, t2 = s_t[new_face], t_t[new_face]
    new_col = torch.div((point * s2).sum(-1) + size - 1, 2, rounding_mode="floor")
    new_row = torch.div((point * t2).sum(-1) + size - 1, 2, rounding_mode="floor")
    return new_face, new_row.clamp(min=0), new_col.clamp(min=0), ~(over_col & over_row)


def _texel_coordinate(coord: Tensor, size: Tensor, shift: float, boundary: str):
    """``coord * size - shift`` wrapped or saturated, and where it is not finite.

    ``reference.py:615-633``: wrapping keeps only the fractional part of ``coord`` first; clamp and
    zero saturate to ``[-1, size]``; non-finite results become 0 and are reported.
    """
    if boundary == "wrap":
        coord = coord - coord.detach().floor()
    x = coord * size - shift
    if boundary in ("clamp", "zero"):
        x = x.clamp(min=-1)
        x = torch.minimum(x, size.to(x.dtype))
    bad = ~torch.isfinite(x)
    return torch.where(bad, 0, x), bad


class _Levels:
    """Mip levels joined into one flat ``[tex_batch * texels, C]`` table with size lookups."""

    def __init__(self, levels: Sequence[Tensor], cube: bool) -> None:
        base = levels[0]
        self.batch = base.shape[0]
        self.channels = base.shape[-1]
        parts, heights, widths, offsets = [], [], [], []
        offset = 0
        for lv in levels:
            lv = lv.expand(self.batch, *lv.shape[1:])
            h, w = lv.shape[-3], lv.shape[-2]
            count = lv.shape[1:-1].numel()
            parts.append(lv.reshape(self.batch, count, self.channels))
            heights.append(h)
            widths.append(w)
            offsets.append(offset)
            offset += count
        self.flat = torch.cat(parts, 1) if len(parts) > 1 else parts[0]
        self.per_batch = offset
        self.heights = torch.tensor(heights)
        self.widths = torch.tensor(widths)
        self.offsets = torch.tensor(offsets)
        self.cube = cube

    def fetch(self, image, level, row, col, boundary, face=None):
        h, w, off = self.heights[level], self.widths[level], self.offsets[level]
        valid = None
        if boundary == "cube":
            face, row, col, valid = cube_fold(face, row, col, w)
        elif boundary == "wrap":
            row, col = torch.remainder(row, h), torch.remainder(col, w)
        else:
            if boundary == "zero":
                valid = (row >= 0) & (row < h) & (col >= 0) & (col < w)
            row = torch.minimum(row.clamp(min=0), h - 1)
            col = torch.minimum(col.clamp(min=0), w - 1)
        if face is not None:
            row = row + face * h
        index = off + row * w + col
        if self.batch > 1:
            index = index + image * self.per_batch
        out = self.flat.reshape(-1, self.channels)[index]
        return out if valid is None else out * valid[..., None]


def _sample_nearest(levels: _Levels, level, uv, boundary, image, face):
    """Texel containing ``uv`` (``reference.py:555-573``)."""
    h, w = levels.heights[level], levels.widths[level]
    x, bad_x = _texel_coordinate(uv[..., 0], w, 0.0, boundary)
    y, bad_y = _texel_coordinate(uv[..., 1], h, 0.0, boundary)
    col, row = x.detach().floor().long(), y.detach().floor().long()
    mode = "clamp" if boundary == "cube" else boundary
    return levels.fetch(image, level, row, col, mode, face), bad_x | bad_y


def _sample_linear(levels: _Levels, level, uv, boundary, image, face):
    """Bilinear blend of four texels, with the cube-corner fill (``reference.py:576-612``)."""
    h, w = levels.heights[level], levels.widths[level]
    x, bad_x = _texel_coordinate(uv[..., 0], w, 0.5, boundary)
    y, bad_y = _texel_coordinate(uv[..., 1], h, 0.5, boundary)
    x0, y0 = x.detach().floor(), y.detach().floor()
    fx, fy = (x - x0)[..., None], (y - y0)[..., None]
    col, row = x0.long(), y0.long()
    taps = [
        levels.fetch(image, level, row + dr, col + dc, boundary, face)
        for dr, dc in ((0, 0), (0, 1), (1, 0), (1, 1))
    ]
    t00, t01, t10, t11 = taps
    out = (1 - fy) * ((1 - fx) * t00 + fx * t01) + fy * ((1 - fx) * t10 + fx * t11)
    if boundary == "cube":
        left, right = (col < 0)[..., None], (col + 1 >= w)[..., None]
        above, below = (row < 0)[..., None], (row + 1 >= h)[..., None]
        missing = (1 - fy) * ((1 - fx) * (left & above) + fx * (right & above)) + fy * (
            (1 - fx) * (left & below) + fx * (right & below)
        )
        out = out + missing * (t00 + t01 + t10 + t11) / 3
    return out, bad_x | bad_y


def texture(
    tex: Tensor,
    uv: Tensor,
    uv_da: Tensor | None = None,
    mip_level_bias: Tensor | None = None,
    mip: Sequence[Tensor] | None = None,
    filter_mode: str = "auto",
    boundary_mode: str = "wrap",
    max_mip_level: int | None = None,
) -> Tensor:
    """Texture lookup with the reference's filtering, boundary and NaN rules.

    ``reference.py:149-194`` and ``ops.py:208-209`` (``auto`` filter). ``mip`` holds levels 1 and
    up; without it the box-filtered chain of ``tex`` is used. Pixels whose coordinates or level of
    detail are not finite are NaN; invalid cube directions read zeros.
    """
    if isinstance(uv_da, Tensor) and uv_da.shape[-1] == 0:
        uv_da = None
    if filter_mode == "auto":
        filter_mode = "linear-mipmap-linear" if (uv_da is not None or mip_level_bias is not None) else "linear"
    mipmapped = "mipmap" in filter_mode
    cube = boundary_mode == "cube"
    face = valid = None
    if cube:
        face, uv, uv_da, valid = cube_project(uv, uv_da if mipmapped else None)
    batch, height, width = uv.shape[:3]
    image = torch.arange(batch)[:, None, None]

    if mipmapped:
        if mip is None:
            chain = mip_chain(tex, max_mip_level)
        else:
            chain = [tex, *mip]
            if max_mip_level is not None:
                chain = chain[: max_mip_level + 1]
        levels = _Levels(chain, cube)
        lod = uv.new_zeros(batch, height, width)
        if uv_da is not None:
            lod = lod + _level_of_detail(uv_da, tex.shape[-3], tex.shape[-2])
        if mip_level_bias is not None:
            lod = lod + mip_level_bias
        top = len(chain) - 1
        bad = lod.isnan()
        lod = torch.where(bad, 0, lod).clamp(0, top)
        blend = filter_mode == "linear-mipmap-linear"
        lower = (lod.detach() + (0.0 if blend else 0.5)).floor().long()
        out, bad_lo = _sample_linear(levels, lower, uv, boundary_mode, image, face)
        bad = bad | bad_lo
        if blend:
            upper = (lower + 1).clamp(max=top)
            frac = (lod - lower)[..., None]
            above, bad_hi = _sample_linear(levels, upper, uv, boundary_mode, image, face)
            out = out * (1 - frac) + above * frac
            bad = bad | bad_hi
    else:
        levels = _Levels([tex], cube)
        level = torch.zeros(batch, height, width, dtype=torch.long)
        sample = _sample_nearest if filter_mode == "nearest" else _sample_linear
        out, bad = sample(levels, level, uv, boundary_mode, image, face)
    out = torch.where(bad[..., None], torch.nan, out)
    return out if valid is None else torch.where(valid[..., None], out, 0)


# --------------------------------------------------------------------------------------------
# Antialiasing
# --------------------------------------------------------------------------------------------


def edge_neighbours(tri: Tensor) -> Tensor:
    """For edge ``3 t + k`` (opposite vertex ``k``), the other edge with the same two vertices.

    ``-1`` when no other edge or more than one other edge uses the vertex pair
    (``reference.py:768-787``). Computed here with a stable sort of 64-bit pair keys in NumPy.
    """
    t = tri.detach().cpu().long().numpy()
    num_edges = 3 * t.shape[0]
    start = t[:, [1, 2, 0]].reshape(-1)
    end = t[:, [2, 0, 1]].reshape(-1)
    key = (np.minimum(start, end) << 32) | np.maximum(start, end)
    order = np.argsort(key, kind="stable")
    sorted_key = key[order]
    out = np.full(num_edges, -1, dtype=np.int64)
    if num_edges:
        boundaries = np.flatnonzero(np.diff(sorted_key)) + 1
        first = np.concatenate([[0], boundaries])
        counts = np.diff(np.concatenate([first, [num_edges]]))
        pairs = first[counts == 2]
        out[order[pairs]] = order[pairs + 1]
        out[order[pairs + 1]] = order[pairs]
    return torch.from_numpy(out).view(-1, 3)


def silhouette_edges(pos: Tensor, tri: Tensor, neighbours: Tensor | None = None) -> Tensor:
    """``[batch, T, 3]``: edge unshared, or shared with a triangle folding over to the same side.

    ``reference.py:790-814``: the side of a vertex ``p`` relative to the projected edge line
    ``l = a x b`` in homogeneous ``(x, y, w)`` is ``sign((l . p) p_w)``.
    """
    pos = pos.detach()
    if pos.ndim == 2:
        pos = pos[None]
    num_tri = tri.shape[0]
    nb = (edge_neighbours(tri) if neighbours is None else neighbours.cpu()).reshape(-1)
    t = tri.long()
    start, end = t[:, [1, 2, 0]].reshape(-1), t[:, [2, 0, 1]].reshape(-1)
    xyw = pos[..., [0, 1, 3]]
    line = torch.linalg.cross(xyw[:, start], xyw[:, end], dim=-1)

    def side(vertex: Tensor) -> Tensor:
        p = xyw[:, vertex]
        return torch.sign((line * p).sum(-1) * p[..., 2])

    opposite = t.reshape(-1)
    shared = nb >= 0
    fold = side(opposite) * side(opposite[nb.clamp(min=0)]) > 0
    return (~shared | fold).view(-1, num_tri, 3)


def _edge_slack(x, y, w, px, py):
    """Rounding bound of each edge function at ``(px, py)`` (``reference.py:730-746``)."""
    a = [x[k] - px * w[k] for k in range(3)]
    c = [y[k] - py * w[k] for k in range(3)]
    rx = [x[k].abs() + w[k].abs() for k in range(3)]
    ry = [y[k].abs() + w[k].abs() for k in range(3)]
    out = []
    for k in range(3):
        i, j = (k + 1) % 3, (k + 2) % 3
        terms = (
            (rx[i] + a[i].abs()) * c[j].abs()
            + (rx[j] + a[j].abs()) * c[i].abs()
            + ry[j] * a[i].abs()
            + ry[i] * a[j].abs()
        )
        out.append(terms * (EDGE_TIE * EPS32))
    return torch.stack(out, -1)


def _crossing(pos3, tri, sil, b, tid, sx, sy, dx, dy, horizontal, height, width):
    """Exit of the triangle at ``src`` towards ``dst``: ``(found, t)`` (``reference.py:675-727``).

    ``t`` is taken from the edge with the smallest crossing among those that ``dst`` lies beyond
    (up to the rounding slack); it counts only when that edge is a silhouette and handled by this
    axis (``reference.py:749-765``).
    """
    n = tid.shape[0]
    cov = (tid >= 0).nonzero().squeeze(1)
    b, tid = b[cov], tid[cov]
    sx, sy, dx, dy = sx[cov], sy[cov], dx[cov], dy[cov]
    pb = b if pos3.shape[0] > 1 else torch.zeros_like(b)
    v = pos3[pb[:, None], tri.long()[tid]]
    x = [v[:, k, 0] for k in range(3)]
    y = [v[:, k, 1] for k in range(3)]
    w = [v[:, k, 3] for k in range(3)]
    e_src = torch.stack(_edge_terms(x, y, w, sx, sy)[2], -1)
    e_dst = torch.stack(_edge_terms(x, y, w, dx, dy)[2], -1)
    sign = torch.where(e_src.sum(-1, keepdim=True) < 0, -1.0, 1.0)
    span = e_src - e_dst
    with torch.no_grad():
        slack = _edge_slack([t.detach() for t in x], [t.detach() for t in y], [t.detach() for t in w], dx, dy)
        crossed = (e_dst * sign <= slack) & (span * sign > 2 * slack)
    t_edge = torch.where(crossed, e_src / torch.where(crossed, span, torch.ones_like(span)), math.inf)
    t, edge = t_edge.min(-1)
    with torch.no_grad():
        xs, ys, ws = (torch.stack([c.detach() for c in comp], -1) for comp in (x, y, w))
        i, j = ((edge + 1) % 3)[:, None], ((edge + 2) % 3)[:, None]
        xi, yi, wi = (s.gather(-1, i).squeeze(-1) for s in (xs, ys, ws))
        xj, yj, wj = (s.gather(-1, j).squeeze(-1) for s in (xs, ys, ws))
        steep = (wj * yi - wi * yj).abs() * height * AXIS_TIE
        flat = (xj * wi - xi * wj).abs() * width
        along = steep >= flat if horizontal else flat > steep
        found = crossed.any(-1) & sil[pb, tid, edge] & along
    all_found = torch.zeros(n, dtype=torch.bool).index_put((cov,), found)
    all_t = t.new_zeros(n).index_put((cov,), torch.where(found, t, 0.0))
    return all_found, all_t


def antialias(
    color: Tensor,
    rast: Tensor,
    pos: Tensor,
    tri: Tensor,
    pos_gradient_boost: float = 1.0,
    neighbours: Tensor | None = None,
) -> Tensor:
    """Silhouette antialiasing by the crossing point of each edge between pixel centres.

    ``reference.py:202-265``. For each right and down pair of pixels with different triangles,
    the crossing ``t`` of the exited silhouette edge is found from each side; the nearer side
    wins when both have one, and the pixel whose half contains the crossing takes ``|t - 1/2|`` of
    the other's colour. Gradients reach ``color`` and, through ``t`` (scaled by
    ``pos_gradient_boost``), ``pos``.
    """
    if tri.shape[0] == 0:
        return color.clone()
    batch, height, width = rast.shape[:3]
    pos3 = pos if pos.ndim == 3 else pos[None]
    tri_id = rast[..., 3].detach().round().long() - 1
    tri_id = torch.where(tri_id < tri.shape[0], tri_id, -1)
    depth = rast[..., 2].detach()
    sil = silhouette_edges(pos3, tri, neighbours)
    px, py = pixel_centres(height, width)
    out = color
    for d_row, d_col in ((0, 1), (1, 0)):
        id_p = tri_id[:, : height - d_row, : width - d_col]
        id_q = tri_id[:, d_row:, d_col:]
        b, r, c = (id_p != id_q).nonzero(as_tuple=True)
        rq, cq = r + d_row, c + d_col
        horizontal = d_col == 1
        found_p, t_p = _crossing(pos3, tri, sil, b, id_p[b, r, c], px[c], py[r], px[cq], py[rq], horizontal, height, width)
        found_q, t_q = _crossing(pos3, tri, sil, b, id_q[b, r, c], px[cq], py[rq], px[c], py[r], horizontal, height, width)
        use_p = found_p & (~found_q | (depth[b, r, c] <= depth[b, rq, cq]))
        use_q = found_q & ~use_p
        t = torch.where(use_p, t_p, 1 - t_q)
        t = t.detach() + pos_gradient_boost * (t - t.detach())
        active = (use_p | use_q)[:, None]
        col_p, col_q = color[b, r, c], color[b, rq, cq]
        delta_p = torch.where(active & (t < 0.5)[:, None], (0.5 - t)[:, None] * (col_q - col_p), 0.0)
        delta_q = torch.where(active & (t >= 0.5)[:, None], (t - 0.5)[:, None] * (col_p - col_q), 0.0)
        out = out.index_put((b, r, c), delta_p, accumulate=True)
        out = out.index_put((b, rq, cq), delta_q, accumulate=True)
    return out.contiguous()
