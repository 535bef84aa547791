"""Generate the golden fixtures by running the reference diffrast package itself.

Run in a container where the reference is importable (its ``src`` directory on ``sys.path``)::

    DIFFRAST_REFERENCE_SRC=<path to diffrast/src> python tests/golden/make_golden.py [maker ...]

Every fixture stores its seeded inputs next to the reference's outputs and gradients (reference
backend, CPU, float32), compressed with NumPy. The tests never import the reference: they read
these files, so they run the same on a machine without it. Scenes come from ``tests/scenes.py``.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))
import scenes  # noqa: E402

SRC = os.environ.get("DIFFRAST_REFERENCE_SRC")
if not SRC:
    raise SystemExit("set DIFFRAST_REFERENCE_SRC to the reference diffrast's src directory")
sys.path.insert(0, SRC)
import diffrast as ref  # noqa: E402
from diffrast.backends import reference as ref_backend  # noqa: E402

ref.set_backend("reference")
torch.set_num_threads(max(1, os.cpu_count() or 1))
CTX = ref.RasterizeContext("cpu")


def save(name: str, **arrays) -> None:
    out = {}
    for key, value in arrays.items():
        if isinstance(value, torch.Tensor):
            value = value.detach().cpu().numpy()
        out[key] = np.asarray(value)
    np.savez_compressed(HERE / f"{name}.npz", **out)
    size = (HERE / f"{name}.npz").stat().st_size
    print(f"{name}: {size / 1024:.1f} KiB")


def raster_case(name, pos, tri, resolution, layers=3, seed=0):
    gen = torch.Generator().manual_seed(seed)
    w_rast = torch.randn(pos.shape[0], *resolution, 4, generator=gen)
    w_db = torch.randn(pos.shape[0], *resolution, 4, generator=gen)
    p = pos.clone().requires_grad_(True)
    rast, rast_db = ref.rasterize(CTX, p, tri, resolution)
    ((rast[..., :3] * w_rast[..., :3]).sum() + (rast_db * w_db).sum()).backward()
    ids = []
    with ref.DepthPeeler(CTX, pos, tri, resolution) as peeler:
        for _ in range(layers):
            r, _ = peeler.rasterize_next_layer()
            ids.append(r[..., 3])
    save(name, pos=pos, tri=tri, resolution=np.array(resolution), w_rast=w_rast, w_db=w_db,
         rast=rast, rast_db=rast_db, grad_pos=p.grad, layer_ids=torch.stack(ids))  # fmt: skip


def make_raster():
    pos, tri = scenes.random_mesh(60, torch.Generator().manual_seed(1), batch=2, w_range=(-1.0, 2.0))
    raster_case("raster_random", pos, tri, (37, 61), seed=11)
    pos, tri = scenes.tiny_mesh(1500, torch.Generator().manual_seed(2), 0.03, batch=2)
    raster_case("raster_tiny", pos, tri, (64, 64), seed=12)
    pos, tri = scenes.grid_mesh(12, torch.Generator().manual_seed(3), batch=2)
    raster_case("raster_grid", pos, tri, (48, 40), seed=13)
    sc = scenes.config1_scene(seed=0)
    raster_case("raster_ico", sc["pos"], sc["tri"], (64, 64), layers=2, seed=14)


def make_interpolate():
    pos, tri = scenes.random_mesh(80, torch.Generator().manual_seed(4), batch=2)
    rast, rast_db = ref.rasterize(CTX, pos, tri, (24, 32))
    gen = torch.Generator().manual_seed(5)
    v = pos.shape[1]
    for layout, shape in (("shared", (v, 6)), ("per_view", (2, v, 6))):
        attr = torch.randn(*shape, generator=gen)
        for tag, diff in (("none", None), ("sel", [3, 0, 5]), ("all", "all")):
            nd = 0 if diff is None else (6 if diff == "all" else 3)
            g_out = torch.randn(2, 24, 32, 6, generator=gen)
            g_da = torch.randn(2, 24, 32, 2 * nd, generator=gen)
            a, r, d = (t.clone().requires_grad_(True) for t in (attr, rast, rast_db))
            out, out_da = ref.interpolate(a, r, tri, rast_db=d, diff_attrs=diff)
            loss = (out * g_out).sum() + (out_da * g_da).sum()
            loss.backward()
            zero = torch.zeros_like
            save(f"interp_{layout}_{tag}", attr=attr, rast=rast, rast_db=rast_db, tri=tri,
                 diff=np.array([] if diff is None else (list(range(6)) if diff == "all" else diff)),
                 g_out=g_out, g_da=g_da, out=out, out_da=out_da,
                 grad_attr=a.grad, grad_rast=r.grad if r.grad is not None else zero(rast),
                 grad_db=d.grad if d.grad is not None else zero(rast_db))  # fmt: skip


FILTERS = ("nearest", "linear", "linear-mipmap-nearest", "linear-mipmap-linear")


def make_texture():
    gen = torch.Generator().manual_seed(6)
    tex = torch.randn(2, 37, 50, 3, generator=gen)
    uv = torch.rand(2, 20, 24, 2, generator=gen) * 1.6 - 0.3
    uv_da = (torch.rand(2, 20, 24, 4, generator=gen) * 0.2 - 0.1) * 4
    bias = torch.rand(2, 20, 24, generator=gen) * 4 - 1
    weights = torch.randn(2, 20, 24, 3, generator=gen)
    for boundary in ("wrap", "clamp", "zero"):
        for fm in FILTERS:
            mip = "mipmap" in fm
            for use_bias in ((False, True) if mip else (False,)):
                t, c, d, bb = (x.clone().requires_grad_(True) for x in (tex, uv, uv_da, bias))
                out = ref.texture(t, c, d if mip else None, mip_level_bias=bb if use_bias else None,
                                  filter_mode=fm, boundary_mode=boundary)  # fmt: skip
                (out.nan_to_num(0) * weights).sum().backward()
                grads = [x.grad if x.grad is not None else torch.zeros_like(x) for x in (t, c, d, bb)]
                tag = f"tex2d_{boundary}_{fm}" + ("_bias" if use_bias else "")
                save(tag, tex=tex, uv=uv, uv_da=uv_da, bias=bias, use_bias=np.array(use_bias),
                     weights=weights, out=out, grad_tex=grads[0], grad_uv=grads[1],
                     grad_uv_da=grads[2], grad_bias=grads[3])  # fmt: skip
    # Non-finite and out-of-range inputs, forward only.
    uv2 = uv.clone()
    uv2[0, 0, :4] = torch.tensor([[float("nan"), 0.5], [float("inf"), 0.2], [-float("inf"), 0.3], [1e30, -1e30]])
    da2 = uv_da.clone()
    da2[0, 1, :3] = torch.tensor([[float("nan"), 0, 0, 0], [float("inf"), 0, 0, 0], [1e30, 1e30, 0, 0]])
    for boundary in ("wrap", "clamp", "zero"):
        out = ref.texture(tex, uv2, da2, filter_mode="linear-mipmap-linear", boundary_mode=boundary)
        save(f"tex2d_edge_{boundary}", tex=tex, uv=uv2, uv_da=da2, out=out)
    # Explicit mip stack with max_mip_level.
    for mml in (0, 2):
        out = ref.texture(tex, uv, uv_da, filter_mode="linear-mipmap-linear", max_mip_level=mml)
        save(f"tex2d_maxmip{mml}", tex=tex, uv=uv, uv_da=uv_da, out=out)
    # The mip chain of odd and even sizes.
    for h, w in ((37, 50), (16, 9), (1, 7)):
        t = torch.randn(1, h, w, 2, generator=gen)
        levels = ref_backend.texture_construct_mip(t, None)
        save(f"mip_{h}x{w}", tex=t, levels=torch.cat([lv.reshape(-1) for lv in levels]))


def make_cube():
    gen = torch.Generator().manual_seed(7)
    tex = torch.randn(1, 6, 16, 16, 3, generator=gen)
    dirs = torch.randn(2, 12, 14, 3, generator=gen)
    dirs_da = torch.randn(2, 12, 14, 6, generator=gen) * 0.05
    weights = torch.randn(2, 12, 14, 3, generator=gen)
    dirs[0, 0, 0] = 0.0
    dirs[0, 0, 1] = torch.tensor([1.0, 1.0, 0.5])
    dirs[0, 0, 2] = torch.tensor([0.3, -0.3, 0.3])
    for fm in FILTERS:
        mip = "mipmap" in fm
        t, d, dd = (x.clone().requires_grad_(True) for x in (tex, dirs, dirs_da))
        out = ref.texture(t, d, dd if mip else None, filter_mode=fm, boundary_mode="cube")
        (out * weights).sum().backward()
        grads = [x.grad if x.grad is not None else torch.zeros_like(x) for x in (t, d, dd)]
        save(f"cube_{fm}", tex=tex, dirs=dirs, dirs_da=dirs_da, weights=weights, out=out,
             grad_tex=grads[0], grad_dirs=grads[1], grad_dirs_da=grads[2])  # fmt: skip


def aa_case(name, pos, tri, resolution, channels, seed, boost=1.0, shared=False):
    gen = torch.Generator().manual_seed(seed)
    rast, _ = ref.rasterize(CTX, pos if not shared else pos.expand(2, -1, -1).contiguous(), tri, resolution)
    batch = rast.shape[0]
    color = torch.rand(batch, *resolution, channels, generator=gen)
    weights = torch.randn(batch, *resolution, channels, generator=gen)
    c = color.clone().requires_grad_(True)
    p_in = pos[0] if shared else pos
    p = p_in.clone().requires_grad_(True)
    out = ref.antialias(c, rast, p, tri, pos_gradient_boost=boost)
    (out * weights).sum().backward()
    sil = ref_backend._silhouette_edges(p_in if p_in.ndim == 3 else p_in[None], tri.long())
    save(name, pos=p_in, tri=tri, rast=rast, color=color, weights=weights, boost=np.array(boost),
         out=out, grad_color=c.grad, grad_pos=p.grad, silhouette=sil,
         neighbours=ref_backend.edge_neighbours(tri))  # fmt: skip


def make_antialias():
    pos, tri = scenes.random_mesh(60, torch.Generator().manual_seed(8), batch=2)
    aa_case("aa_random", pos, tri, (48, 64), 3, seed=21)
    aa_case("aa_random_boost", pos, tri, (48, 64), 2, seed=22, boost=2.5)
    pos, tri = scenes.grid_mesh(10, torch.Generator().manual_seed(9), batch=2)
    aa_case("aa_grid", pos, tri, (40, 48), 3, seed=23)
    sc = scenes.config1_scene(seed=0)
    aa_case("aa_ico", sc["pos"], sc["tri"], (64, 64), 3, seed=24)
    pos, tri = scenes.random_mesh(40, torch.Generator().manual_seed(10), batch=1, w_range=(-1.0, 2.0))
    aa_case("aa_shared", pos, tri, (32, 40), 1, seed=25, shared=True)


def make_topology():
    verts, tri = scenes.icosphere(2)
    nb = ref_backend.edge_neighbours(tri)
    # A non-manifold fan: three triangles on one edge, plus a duplicate triangle.
    extra = torch.tensor([[0, 1, 2], [1, 0, 3], [0, 1, 4], [5, 6, 7], [5, 6, 7]], dtype=torch.int32)
    nb2 = ref_backend.edge_neighbours(extra)
    save("topology", tri=tri, neighbours=nb, tri_fan=extra, neighbours_fan=nb2)


def make_bench_scene():
    """The displaced grid of the reference's benchmarks (``benchmarks/bench_rasterize.py``, next
    to ``src``), which ``scenes.displaced_grid`` restates for ``bench_configs.py``."""
    sys.path.insert(0, str(Path(SRC).resolve().parent / "benchmarks"))
    from bench_rasterize import grid_mesh

    pos, tri = grid_mesh(200, 3, torch.device("cpu"))
    n = round((pos.shape[1]) ** 0.5) - 1
    steps = torch.linspace(0, 1, n + 1)
    uv = torch.stack(torch.meshgrid(steps, steps, indexing="xy"), -1).reshape(-1, 2)
    save("bench_grid", num_tri=np.array(200), views=np.array(3), pos=pos, tri=tri, uv=uv)


MAKERS = {"raster": make_raster, "interpolate": make_interpolate, "texture": make_texture,
          "cube": make_cube, "antialias": make_antialias, "topology": make_topology,
          "bench_scene": make_bench_scene}  # fmt: skip

if __name__ == "__main__":
    # python make_golden.py [maker ...]: all fixtures, or only the named makers'.
    for name in sys.argv[1:] or MAKERS:
        MAKERS[name]()
