"""BASELINE configurations 2-5 at reduced size: the CUDA path against the CPU oracle end to end.

Each test runs the configuration's op sequence (scenes.config*_small: the same generators and
parameters with fewer views, triangles and pixels) on both devices and compares triangle ids
exactly, forward values within rel 1e-4 (looser after long chains, stated per check) and
gradients within the atomic-accumulation tolerance.
"""

import pytest
import torch

import diffrast_b200 as dr
import oracle
import scenes

pytestmark = pytest.mark.gpu
CUDA = "cuda"


def close(a, b, tol):
    scale = max(1.0, b.abs().max().item()) if b.numel() else 1.0
    torch.testing.assert_close(a.detach().cpu(), b.detach().cpu(), atol=tol * scale, rtol=tol,
                               equal_nan=True)


@pytest.fixture(scope="module")
def ctx():
    return dr.RasterizeContext(CUDA)


def test_config2_rasterize_only(ctx):
    sc = scenes.config2_small()
    results = []
    for dev in ("cpu", CUDA):
        pos = sc["pos"].to(dev).clone().requires_grad_(True)
        tri = sc["tri"].to(dev)
        if dev == "cpu":
            rast, rast_db = oracle.rasterize(pos, tri, sc["resolution"])
        else:
            rast, rast_db = dr.rasterize(ctx, pos, tri, sc["resolution"])
        ((rast * sc["g_rast"].to(dev)).sum() + (rast_db * sc["g_db"].to(dev)).sum()).backward()
        results.append((rast, rast_db, pos.grad))
    (ref_rast, ref_db, ref_g), (rast, rast_db, g) = results
    assert torch.equal(rast[..., 3].cpu(), ref_rast[..., 3]), "triangle ids"
    close(rast[..., :3], ref_rast[..., :3], 1e-4)
    close(rast_db, ref_db, 1e-3)
    close(g, ref_g, 1e-3)


def test_config3_attributes_and_mip_stack(ctx):
    sc = scenes.config3_small()
    results = []
    for dev in ("cpu", CUDA):
        pos = sc["pos"].to(dev).clone().requires_grad_(True)
        attr = sc["attr"].to(dev).clone().requires_grad_(True)
        tex = sc["tex"].to(dev).clone().requires_grad_(True)
        tri = sc["tri"].to(dev)
        diff = list(range(attr.shape[-1]))
        if dev == "cpu":
            rast, rast_db = oracle.rasterize(pos, tri, sc["resolution"])
            out, out_da = oracle.interpolate(attr, rast, tri, rast_db, diff)
            color = oracle.texture(tex, out[..., 0:2], out_da[..., 0:4], None, None,
                                   "linear-mipmap-linear", "wrap")
        else:
            rast, rast_db = dr.rasterize(ctx, pos, tri, sc["resolution"])
            out, out_da = dr.interpolate(attr, rast, tri, rast_db=rast_db, diff_attrs="all")
            stack = dr.texture_construct_mip(tex)
            color = dr.texture(tex, out[..., 0:2], out_da[..., 0:4], mip=stack,
                               filter_mode="linear-mipmap-linear")
        loss = ((color - sc["target"].to(dev)) ** 2).mean() + (out[..., 2:] ** 2).mean()
        loss.backward()
        results.append((rast, color, pos.grad, attr.grad, tex.grad))
    ref, ours = results
    assert torch.equal(ours[0][..., 3].cpu(), ref[0][..., 3]), "triangle ids"
    close(ours[1], ref[1], 1e-4)
    for i in (2, 3, 4):  # pos, attr, tex gradients
        close(ours[i], ref[i], 2e-3)


def test_config4_cube_peeling_antialias(ctx):
    sc = scenes.config4_small()
    results = []
    for dev in ("cpu", CUDA):
        pos = sc["pos"].to(dev).clone().requires_grad_(True)
        cube = sc["cube"].to(dev).clone().requires_grad_(True)
        tri, normals = sc["tri"].to(dev), sc["normals"].to(dev)
        target = sc["target"].to(dev)
        ids, images, loss = [], [], 0.0
        peeler = dr.DepthPeeler(ctx, pos, tri, sc["resolution"]) if dev == CUDA else None
        state = None
        for _ in range(sc["layers"]):
            if dev == "cpu":
                rast, rast_db, state = oracle.rasterize_layer(pos, tri, sc["resolution"], True, state)
                n, n_da = oracle.interpolate(normals, rast, tri, rast_db, [0, 1, 2])
                color = oracle.texture(cube, n, n_da, None, None, "linear-mipmap-linear", "cube")
                image = oracle.antialias(color, rast, pos, tri)
            else:
                rast, rast_db = peeler.rasterize_next_layer()
                n, n_da = dr.interpolate(normals, rast, tri, rast_db=rast_db, diff_attrs="all")
                color = dr.texture(cube, n, n_da, filter_mode="linear-mipmap-linear",
                                   boundary_mode="cube")
                image = dr.antialias(color, rast, pos, tri)
            ids.append(rast[..., 3].detach().cpu())
            images.append(image)
            loss = loss + ((image - target) ** 2).mean()
        loss.backward()
        results.append((ids, images, pos.grad, cube.grad))
    ref, ours = results
    for layer, (a, b) in enumerate(zip(ours[0], ref[0])):
        assert torch.equal(a, b), f"triangle ids of layer {layer}"
    for a, b in zip(ours[1], ref[1]):
        close(a, b, 1e-4)
    close(ours[2], ref[2], 2e-3)
    close(ours[3], ref[3], 2e-3)


def test_config5_spiky_mesh_pipeline(ctx):
    """The hot path's own workload character: triangles about a pixel wide whose displacement
    exceeds their size, overlapping several deep (ties and near-ties everywhere)."""
    sc = scenes.config5_small()
    results = []
    for dev in ("cpu", CUDA):
        pos = sc["pos"].to(dev).clone().requires_grad_(True)
        tex = sc["tex"].to(dev).clone().requires_grad_(True)
        tri, attr = sc["tri"].to(dev), sc["attr"].to(dev)
        if dev == "cpu":
            rast, rast_db = oracle.rasterize(pos, tri, sc["resolution"])
            out, out_da = oracle.interpolate(attr, rast, tri, rast_db, list(range(5)))
            color = oracle.texture(tex, out[..., 0:2], out_da[..., 0:4], None, None,
                                   "linear-mipmap-linear", "wrap")
            image = oracle.antialias(color, rast, pos, tri)
        else:
            rast, rast_db = dr.rasterize(ctx, pos, tri, sc["resolution"])
            out, out_da = dr.interpolate(attr, rast, tri, rast_db=rast_db, diff_attrs="all")
            color = dr.texture(tex, out[..., 0:2], out_da[..., 0:4],
                               filter_mode="linear-mipmap-linear")
            image = dr.antialias(color, rast, pos, tri)
        torch.nn.functional.mse_loss(image, sc["target"].to(dev), reduction="sum").backward()
        blended = (image != color).detach().cpu()
        results.append((rast, image, pos.grad, tex.grad, blended))
    ref, ours = results
    assert torch.equal(ours[0][..., 3].cpu(), ref[0][..., 3]), "triangle ids"
    assert torch.equal(ours[4], ref[4]), "antialias edge set (blended pixels)"
    close(ours[1], ref[1], 1e-4)
    close(ours[2], ref[2], 2e-3)
    close(ours[3], ref[3], 2e-3)
