"""Lambert shading (``dr.lambert``) against a plain PyTorch float32 restatement of the same
formula, forward and backward: ``color * (ambient + max(0, n . l))`` with unit normal and light,
zero normals shading with the ambient term alone. Tolerances: values rel 1e-5 / abs 1e-6,
gradients rel 1e-4 / abs 1e-5 (scaled by the largest gradient)."""

import pytest
import torch

import diffrast_b200 as dr
import scenes

pytestmark = pytest.mark.gpu
CUDA = "cuda"


def torch_lambert(color, normal, light, ambient):
    norm = normal.norm(dim=-1, keepdim=True)
    unit = torch.where(norm > 0, normal / norm.clamp_min(1e-30), torch.zeros_like(normal))
    l = light.reshape(-1, 3)
    l = l / l.norm(dim=-1, keepdim=True)
    d = (unit * l[:, None, None, :]).sum(-1, keepdim=True).clamp_min(0.0)
    return color * (ambient + d)


def close(a, b, rtol, atol):
    scale = max(1.0, b.abs().max().item())
    torch.testing.assert_close(a, b, rtol=rtol, atol=atol * scale)


@pytest.mark.parametrize("per_view_light", [False, True])
def test_lambert_matches_torch(per_view_light):
    gen = torch.Generator().manual_seed(3)
    color = torch.rand(3, 20, 24, 3, generator=gen)
    normal = torch.randn(3, 20, 24, 3, generator=gen)
    normal[:, :4] = 0.0  # background rows
    light = torch.randn(3 if per_view_light else 1, 3, generator=gen)
    light = light if per_view_light else light[0]
    weights = torch.randn(3, 20, 24, 3, generator=gen)
    results = []
    for dev in ("cpu", CUDA):
        c = color.detach().clone().to(dev).requires_grad_(True)
        n = normal.detach().clone().to(dev).requires_grad_(True)
        lt = light.to(dev)
        out = torch_lambert(c, n, lt, 0.2) if dev == "cpu" else dr.lambert(c, n, lt, ambient=0.2)
        (out * weights.to(dev)).sum().backward()
        results.append((out.detach().cpu(), c.grad.cpu(), n.grad.cpu()))
    ref, ours = results
    torch.testing.assert_close(ours[0], ref[0], rtol=1e-5, atol=1e-6)
    close(ours[1], ref[1], 1e-4, 1e-5)
    close(ours[2], ref[2], 1e-4, 1e-5)
    assert (ours[2][:, :4] == 0).all()


def test_lambert_of_interpolated_normals_in_place():
    """Normals as a channel slice of interpolate's output (read with its pixel stride); the
    normal gradient reaches the attributes through the interpolation."""
    sc = scenes.config5_small(views=2)
    ctx = dr.RasterizeContext(CUDA)
    pos, tri = sc["pos"].cuda(), sc["tri"].cuda()
    gen = torch.Generator().manual_seed(5)
    color0 = torch.rand(2, 64, 64, 3, generator=gen).cuda()
    light = torch.tensor([0.3, 0.5, 0.8], device=CUDA)
    rast, rast_db = dr.rasterize(ctx, pos, tri, sc["resolution"])
    results = []
    for ours in (True, False):
        attr = sc["attr"].cuda().requires_grad_(True)
        color = color0.clone().requires_grad_(True)
        out, _ = dr.interpolate(attr, rast, tri)
        normal = out[..., 2:5]
        shaded = dr.lambert(color, normal, light) if ours else torch_lambert(color, normal, light, 0.0)
        (shaded ** 2).sum().backward()
        results.append((shaded.detach(), attr.grad, color.grad))
    for a, b in zip(*results):
        close(a.cpu(), b.cpu(), 1e-4, 1e-5)
