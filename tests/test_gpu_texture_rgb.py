"""Three-channel lookups take their own kernel variants (the channel count a template argument, so
that the channel loops unroll and all texel gathers of a pixel are in flight together). The same
lookup on the texture padded with a zero fourth channel takes the generic variants, whose
arithmetic per channel is the same: values must agree bit for bit, and gradients (texel gradients
are float atomics, accumulated in any order) within float32 rounding."""

import pytest
import torch

import diffrast_b200 as dr

pytestmark = pytest.mark.gpu
CUDA = "cuda"


def _inputs(seed, views, res, tex_size):
    gen = torch.Generator().manual_seed(seed)
    tex = torch.rand(1, tex_size, tex_size, 3, generator=gen)
    # Coordinates spread over and beyond [0, 1] (wrapping and clamping both matter) with
    # footprints from magnified to minified, so that every level pair is used.
    uv = torch.rand(views, res, res, 2, generator=gen) * 1.6 - 0.3
    scale = torch.exp2(torch.rand(views, res, res, 1, generator=gen) * 10.0 - 8.0)
    uv_da = torch.randn(views, res, res, 4, generator=gen) * scale
    grad = torch.randn(views, res, res, 3, generator=gen)
    return [t.to(CUDA) for t in (tex, uv, uv_da, grad)]


def _lookup(tex, uv, uv_da, grad, filter_mode, boundary_mode):
    tex = tex.detach().requires_grad_(True)
    uv = uv.detach().requires_grad_(True)
    # Plain bilinear lookups take no footprint.
    uv_da = uv_da.detach().requires_grad_(True) if filter_mode != "linear" else None
    out = dr.texture(tex, uv, uv_da, filter_mode=filter_mode, boundary_mode=boundary_mode)
    channels = grad.shape[-1]
    (out[..., :channels] * grad).sum().backward()
    g_da = uv_da.grad if uv_da is not None else torch.zeros(0, device=CUDA)
    return out.detach(), tex.grad, uv.grad, g_da


@pytest.mark.parametrize("filter_mode", ["linear", "linear-mipmap-nearest", "linear-mipmap-linear"])
@pytest.mark.parametrize("boundary_mode", ["wrap", "clamp", "zero"])
def test_rgb_variants_match_generic(filter_mode, boundary_mode):
    tex, uv, uv_da, grad = _inputs(7, views=2, res=48, tex_size=64)
    padded = torch.cat([tex, torch.zeros_like(tex[..., :1])], dim=-1)
    out3, gtex3, guv3, gda3 = _lookup(tex, uv, uv_da, grad, filter_mode, boundary_mode)
    out4, gtex4, guv4, gda4 = _lookup(padded, uv, uv_da, grad, filter_mode, boundary_mode)
    assert torch.equal(out3, out4[..., :3])
    # The compiler may contract products and sums differently in the unrolled loops: gradients
    # within float32 rounding.
    torch.testing.assert_close(guv3, guv4, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(gda3, gda4, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(gtex3, gtex4[..., :3], rtol=1e-5, atol=1e-6)
    assert torch.count_nonzero(gtex4[..., 3]) == 0
