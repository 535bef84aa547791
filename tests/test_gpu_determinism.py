"""Determinism: the same inputs give bit-identical visibility keys, triangle ids, rast, rast_db,
interpolated attributes, texture lookups and antialiased images on every run (64-bit atomic
minima and pixel-owned writes are order-independent); gradients, accumulated with float atomics
in whatever order the hardware runs them, agree within 1e-5 relative to the largest value."""

import pytest
import torch

import diffrast_b200 as dr
import scenes
from diffrast_b200 import ops

pytestmark = pytest.mark.gpu
CUDA = "cuda"


def run(sc, ctx):
    pos = sc["pos"].cuda().requires_grad_(True)
    tex = sc["tex"].cuda().requires_grad_(True)
    tri, attr, target = sc["tri"].cuda(), sc["attr"].cuda(), sc["target"].cuda()
    rast, rast_db, keys = ops.rasterize_layer(pos, tri, sc["resolution"], True, None)
    out, out_da = dr.interpolate(attr, rast, tri, rast_db=rast_db, diff_attrs="all")
    color = dr.texture(tex, out[..., 0:2], out_da[..., 0:4], filter_mode="linear-mipmap-linear")
    image, loss = dr.antialias_mse(color, rast, pos, tri, target)
    loss.backward()
    return dict(keys=keys, rast=rast.detach(), rast_db=rast_db.detach(), out=out.detach(),
                color=color.detach(), image=image.detach(), g_pos=pos.grad, g_tex=tex.grad)


@pytest.mark.parametrize("views,resolution,subdivisions", [(2, 64, 4), (4, 256, 6)])
def test_runs_agree(views, resolution, subdivisions):
    sc = scenes.config5_small(views=views, resolution=resolution, subdivisions=subdivisions,
                              noise=0.15 / 2 ** (subdivisions - 4))
    ctx = dr.RasterizeContext(CUDA)
    first, second = run(sc, ctx), run(sc, ctx)
    assert (first["rast"][..., 3] > 0).any()
    for key in ("keys", "rast", "rast_db", "out", "color", "image"):
        assert torch.equal(first[key], second[key]), key
    for key in ("g_pos", "g_tex"):
        scale = max(1.0, first[key].abs().max().item())
        torch.testing.assert_close(second[key], first[key], atol=1e-5 * scale, rtol=1e-5)
