"""antialias_mse: antialias with the squared-error loss fused into its kernels, against the
unfused composition (antialias, then torch's mse_loss) and against the CPU oracle.

Tolerances: the image is the same kernel arithmetic (bit-exact); the loss rel 1e-5 (block partial
sums in float32 against torch's reduction); gradients rel/abs 1e-3 scaled by the largest value
(atomic accumulation order).
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
    torch.testing.assert_close(a.detach().cpu(), b.detach().cpu(), atol=tol * scale, rtol=tol)


@pytest.fixture(scope="module")
def scene():
    sc = scenes.config5_small()
    ctx = dr.RasterizeContext(CUDA)
    pos = sc["pos"].to(CUDA)
    tri = sc["tri"].to(CUDA)
    rast, _ = dr.rasterize(ctx, pos, tri, sc["resolution"])
    gen = torch.Generator().manual_seed(21)
    color = torch.rand(*rast.shape[:3], 3, generator=gen).to(CUDA)
    target = torch.rand(*rast.shape[:3], 3, generator=gen).to(CUDA)
    return pos, tri, rast, color, target


def run(fused, pos, tri, rast, color, target, scale=None, extra=None):
    p = pos.clone().requires_grad_(True)
    c = color.clone().requires_grad_(True)
    if fused:
        image, loss = dr.antialias_mse(c, rast, p, tri, target, scale=scale)
    else:
        image = dr.antialias(c, rast, p, tri)
        s = 1.0 / image.numel() if scale is None else scale
        loss = ((image - target) ** 2).sum() * s
    total = loss if extra is None else loss + (image * extra).sum()
    total.backward()
    return image, loss, c.grad, p.grad


@pytest.mark.parametrize("scale", [None, 0.37])
def test_fused_matches_unfused(scene, scale):
    ours = run(True, *scene, scale=scale)
    ref = run(False, *scene, scale=scale)
    assert torch.equal(ours[0], ref[0]), "image"
    torch.testing.assert_close(ours[1], ref[1], rtol=1e-5, atol=0)
    close(ours[2], ref[2], 1e-3)
    close(ours[3], ref[3], 1e-3)


def test_fused_adds_gradients_reaching_the_image(scene):
    extra = torch.randn(scene[3].shape, generator=torch.Generator().manual_seed(2)).to(CUDA)
    ours = run(True, *scene, extra=extra)
    ref = run(False, *scene, extra=extra)
    close(ours[2], ref[2], 1e-3)
    close(ours[3], ref[3], 1e-3)


def test_fused_matches_oracle(scene):
    pos, tri, rast, color, target = scene
    image, loss, g_color, g_pos = run(True, pos, tri, rast, color, target)
    p = pos.cpu().clone().requires_grad_(True)
    c = color.cpu().clone().requires_grad_(True)
    ref = oracle.antialias(c, rast.cpu(), p, tri.cpu())
    ref_loss = torch.nn.functional.mse_loss(ref, target.cpu())
    ref_loss.backward()
    close(image, ref, 1e-4)
    torch.testing.assert_close(loss.cpu(), ref_loss.detach(), rtol=1e-5, atol=0)
    close(g_color, c.grad, 1e-3)
    close(g_pos, p.grad, 1e-3)


def test_fused_without_triangles():
    color = torch.rand(1, 8, 8, 3, device=CUDA, requires_grad=True)
    target = torch.zeros(1, 8, 8, 3, device=CUDA)
    rast = torch.zeros(1, 8, 8, 4, device=CUDA)
    pos = torch.zeros(1, 3, 4, device=CUDA)
    image, loss = dr.antialias_mse(color, rast, pos, torch.zeros(0, 3, dtype=torch.int32, device=CUDA), target)
    loss.backward()
    assert torch.equal(image, color.detach())
    torch.testing.assert_close(loss, (color.detach() ** 2).mean(), rtol=1e-5, atol=0)
    torch.testing.assert_close(color.grad, 2 * color.detach() / color.numel(), rtol=1e-5, atol=1e-8)
