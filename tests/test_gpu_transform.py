"""World-to-clip transform kernels against a float64 PyTorch restatement of diffrast's
examples/common.py:320-323 (homogeneous positions times the transposed matrices).

Tolerances: forward rel 1e-5 (a few float32 roundings of a 4-term dot product); gradients rel
1e-4 scaled by the largest value (sums over up to 70 views and 10^5 vertices in float32).
"""

import pytest
import torch

import diffrast_b200 as dr

pytestmark = pytest.mark.gpu


def reference(positions, matrix):
    homogeneous = torch.nn.functional.pad(positions, (0, 1), value=1.0)
    return homogeneous @ matrix.transpose(-1, -2)


def close(a, b, tol):
    scale = max(1.0, b.abs().max().item()) if b.numel() else 1.0
    torch.testing.assert_close(a.detach().cpu().double(), b.detach().cpu().double(),
                               atol=tol * scale, rtol=tol)


@pytest.mark.parametrize("views, vertices", [(1, 3), (5, 1000), (70, 4099), (64, 100_003)])
def test_to_clip_forward_and_gradients(views, vertices):
    gen = torch.Generator().manual_seed(views * 7 + vertices)
    positions = torch.randn(vertices, 3, generator=gen)
    matrix = torch.randn(views, 4, 4, generator=gen)
    upstream = torch.randn(views, vertices, 4, generator=gen)

    p = positions.cuda().requires_grad_(True)
    m = matrix.cuda().requires_grad_(True)
    clip = dr.to_clip(p, m)
    (clip * upstream.cuda()).sum().backward()

    p64 = positions.double().requires_grad_(True)
    m64 = matrix.double().requires_grad_(True)
    ref = reference(p64, m64)
    (ref * upstream.double()).sum().backward()

    assert clip.shape == (views, vertices, 4)
    close(clip, ref, 1e-5)
    close(p.grad, p64.grad, 1e-4)
    close(m.grad, m64.grad, 1e-4)


def test_to_clip_only_positions_need_gradients():
    gen = torch.Generator().manual_seed(3)
    p = torch.randn(500, 3, generator=gen).cuda().requires_grad_(True)
    m = torch.randn(4, 4, 4, generator=gen).cuda()
    dr.to_clip(p, m).square().sum().backward()
    assert m.grad is None and p.grad is not None
    ref_p = p.detach().cpu().double().requires_grad_(True)
    reference(ref_p, m.cpu().double()).square().sum().backward()
    close(p.grad, ref_p.grad, 1e-4)


def test_to_clip_empty_and_feeds_the_rasterizer():
    m = torch.eye(4).repeat(2, 1, 1).cuda()
    assert dr.to_clip(torch.zeros(0, 3, device="cuda"), m).shape == (2, 0, 4)
    tri_pos = torch.tensor([[-0.5, -0.5, 0.0], [0.5, -0.5, 0.0], [0.0, 0.5, 0.0]], device="cuda")
    clip = dr.to_clip(tri_pos, m)
    rast, _ = dr.rasterize(dr.RasterizeContext("cuda"), clip,
                           torch.tensor([[0, 1, 2]], dtype=torch.int32, device="cuda"), (16, 16))
    assert (rast[..., 3] == 1).sum() > 0
