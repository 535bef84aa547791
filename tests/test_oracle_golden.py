"""The CPU oracle reproduces the reference package's own outputs (golden fixtures).

These pin the restatement in ``oracle/`` before it is trusted as the checker of the CUDA kernels.
Triangle ids, silhouettes and edge adjacency must be identical; floats agree to float32 rounding.
"""

import pytest
import torch

import oracle
from conftest import golden_names, load_golden


def close(a, b, tol=1e-5):
    torch.testing.assert_close(a, b, atol=tol, rtol=tol, equal_nan=True)


@pytest.mark.parametrize("name", golden_names("raster_"))
def test_rasterize_matches_reference(name):
    g = load_golden(name)
    res = tuple(g["resolution"].tolist())
    p = g["pos"].clone().requires_grad_(True)
    rast, rast_db = oracle.rasterize(p, g["tri"], res)
    assert torch.equal(rast[..., 3], g["rast"][..., 3]), "triangle ids must be bit-exact"
    close(rast, g["rast"])
    close(rast_db, g["rast_db"], 1e-4)
    ((rast[..., :3] * g["w_rast"][..., :3]).sum() + (rast_db * g["w_db"]).sum()).backward()
    scale = g["grad_pos"].abs().max().item()
    close(p.grad, g["grad_pos"], 1e-4 * max(1.0, scale))
    state = None
    for k in range(g["layer_ids"].shape[0]):
        r, _, state = oracle.rasterize_layer(g["pos"], g["tri"], res, True, state)
        assert torch.equal(r[..., 3], g["layer_ids"][k]), f"layer {k}"


@pytest.mark.parametrize("name", golden_names("interp_"))
def test_interpolate_matches_reference(name):
    g = load_golden(name)
    diff = g["diff"].long().tolist()
    a, r, d = (g[k].clone().requires_grad_(True) for k in ("attr", "rast", "rast_db"))
    out, out_da = oracle.interpolate(a, r, g["tri"], d, diff)
    close(out, g["out"])
    close(out_da, g["out_da"])
    ((out * g["g_out"]).sum() + (out_da * g["g_da"]).sum()).backward()
    close(a.grad, g["grad_attr"], 1e-4)
    close(r.grad, g["grad_rast"], 1e-4)
    close(d.grad if d.grad is not None else torch.zeros_like(d), g["grad_db"], 1e-4)


@pytest.mark.parametrize("name", [n for n in golden_names("tex2d_") if "edge" not in n and "maxmip" not in n])
def test_texture_matches_reference(name):
    g = load_golden(name)
    boundary, mode = name.split("_")[1], name.split("_")[2]
    mip = "mipmap" in mode
    use_bias = bool(g["use_bias"].item())
    t, c, d, bb = (g[k].clone().requires_grad_(True) for k in ("tex", "uv", "uv_da", "bias"))
    out = oracle.texture(t, c, d if mip else None, bb if use_bias else None, None, mode, boundary)
    close(out, g["out"])
    (out.nan_to_num(0) * g["weights"]).sum().backward()
    for x, key in ((t, "grad_tex"), (c, "grad_uv"), (d, "grad_uv_da"), (bb, "grad_bias")):
        grad = x.grad if x.grad is not None else torch.zeros_like(x)
        close(grad, g[key], 1e-3)


@pytest.mark.parametrize("boundary", ["wrap", "clamp", "zero"])
def test_texture_non_finite_inputs_match_reference(boundary):
    g = load_golden(f"tex2d_edge_{boundary}")
    out = oracle.texture(g["tex"], g["uv"], g["uv_da"], None, None, "linear-mipmap-linear", boundary)
    close(out, g["out"])


@pytest.mark.parametrize("level", [0, 2])
def test_texture_max_mip_level_matches_reference(level):
    g = load_golden(f"tex2d_maxmip{level}")
    out = oracle.texture(g["tex"], g["uv"], g["uv_da"], None, None, "linear-mipmap-linear", "wrap", level)
    close(out, g["out"])


@pytest.mark.parametrize("name", golden_names("mip_"))
def test_mip_chain_matches_reference(name):
    g = load_golden(name)
    levels = oracle.mip_chain(g["tex"])[1:]
    close(torch.cat([lv.reshape(-1) for lv in levels]), g["levels"])


@pytest.mark.parametrize("name", golden_names("cube_"))
def test_cube_texture_matches_reference(name):
    g = load_golden(name)
    mode = name[len("cube_"):]
    mip = "mipmap" in mode
    t, d, dd = (g[k].clone().requires_grad_(True) for k in ("tex", "dirs", "dirs_da"))
    out = oracle.texture(t, d, dd if mip else None, None, None, mode, "cube")
    close(out, g["out"])
    (out * g["weights"]).sum().backward()
    for x, key in ((t, "grad_tex"), (d, "grad_dirs"), (dd, "grad_dirs_da")):
        grad = x.grad if x.grad is not None else torch.zeros_like(x)
        close(grad, g[key], 1e-3)


@pytest.mark.parametrize("name", golden_names("aa_"))
def test_antialias_matches_reference(name):
    g = load_golden(name)
    sil = oracle.silhouette_edges(g["pos"], g["tri"])
    assert torch.equal(sil, g["silhouette"]), "silhouette edge set must be bit-exact"
    assert torch.equal(oracle.edge_neighbours(g["tri"]), g["neighbours"])
    c = g["color"].clone().requires_grad_(True)
    p = g["pos"].clone().requires_grad_(True)
    out = oracle.antialias(c, g["rast"], p, g["tri"], float(g["boost"]))
    close(out, g["out"])
    (out * g["weights"]).sum().backward()
    close(c.grad, g["grad_color"], 1e-5)
    scale = g["grad_pos"].abs().max().item()
    close(p.grad, g["grad_pos"], 1e-4 * max(1.0, scale))


def test_edge_neighbours_match_reference():
    g = load_golden("topology")
    assert torch.equal(oracle.edge_neighbours(g["tri"]), g["neighbours"])
    assert torch.equal(oracle.edge_neighbours(g["tri_fan"]), g["neighbours_fan"])


def test_keys_order_like_depth_then_index():
    depth = torch.tensor([[-0.5, -0.0, 0.0, 0.25, 0.25, 1.0]])
    ids = torch.tensor([[7, 3, 2, 9, 4, 0]])
    keys = oracle.keys_from_state(depth, ids)
    order = keys.argsort(-1)
    assert order.tolist() == [[0, 2, 1, 4, 3, 5]]
    assert oracle.keys_from_state(depth, torch.full_like(ids, -1)).eq(oracle.EMPTY_KEY).all()
