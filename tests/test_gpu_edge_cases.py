"""Edge cases the reference tests, on the CUDA path.

- Very wide and very tall images (2 x 80001 up to 200003 x 2 pixels): quads whose opposite sides
  lie exactly on pixel-centre columns (rows), so the conservative pixel bounds of the visibility
  pass must keep them despite the rounding of x / w, which grows with the image size (reference
  tests/test_coverage.py:766-790). Coverage must equal the fill rule's exact answer; the resolve,
  interpolation and antialias passes (launched in row chunks above 65535 rows) run on them too.
- Level of detail of very long textures, 46342 and 65536 texels long (tests/test_mip.py:586-600):
  stripes of zeros and ones average to one half from the first mip level on.
- rast_db against finite differences of rast under sub-pixel shifts
  (tests/test_gradients.py:60-75).
- The antialias position gradient against float64 finite differences of the oracle's antialiased
  image (tests/test_antialias.py:165-220): a constant-colour triangle, interpolated colours and two
  overlapping triangles.

Tolerances are stated per test.
"""

import pytest
import torch

import diffrast_b200 as dr
import oracle

pytestmark = pytest.mark.gpu
CUDA = "cuda"
QUAD = torch.tensor([[0, 1, 2], [0, 2, 3]], dtype=torch.int32)


@pytest.fixture(scope="module")
def ctx():
    return dr.RasterizeContext(CUDA)


def lattice(cols, rows, resolution):
    """Clip-space vertices (w = 1) exactly on the centres of pixels (rows, cols)."""
    height, width = resolution
    x = (cols.float() * 2 + 1) / width - 1
    y = (rows.float() * 2 + 1) / height - 1
    return torch.stack([x, y, torch.zeros_like(x), torch.ones_like(x)], -1)[None]


def perspective_triangle():
    pos = torch.tensor([[[-0.8, -0.6, 0.2, 1.0], [1.2, -0.9, 0.5, 2.0], [0.1, 1.5, -0.3, 1.5]]])
    return pos, torch.tensor([[0, 1, 2]], dtype=torch.int32)


@pytest.mark.parametrize("size", [80001, 200003])
@pytest.mark.parametrize("tall", [False, True])
def test_very_wide_and_very_tall_images(ctx, size, tall):
    """Coverage equals the exact fill-rule answer: pixel i is covered by a quad spanning the
    centres of pixels first .. last iff first <= i < last (its right edge, through centres,
    belongs to the next pixel by the top-left rule). Ids at sampled pixels equal the oracle's."""
    gen = torch.Generator().manual_seed(8)
    first = torch.randint(0, size - 8, (3000,), generator=gen)
    last = first + torch.randint(1, 4, (3000,), generator=gen)
    along = torch.stack([first, last, last, first], -1).flatten()
    across = torch.tensor([-2, -2, 4, 4]).repeat(3000)
    resolution = (size, 2) if tall else (2, size)
    cols, rows = (across, along) if tall else (along, across)
    pos_cpu = lattice(cols, rows, resolution)
    tri_cpu = (QUAD[None] + torch.arange(3000)[:, None, None] * 4).view(-1, 3).int()
    edges = torch.zeros(size + 1)
    edges.index_add_(0, first, torch.ones(3000)).index_add_(0, last, -torch.ones(3000))
    expected = (edges.cumsum(0)[:size] > 0).expand(2, size)

    pos = pos_cpu.cuda().requires_grad_(True)
    tri = tri_cpu.cuda()
    rast, rast_db = dr.rasterize(ctx, pos, tri, resolution)
    covered = (rast[0, ..., 3] > 0).cpu()
    assert torch.equal(covered.T if tall else covered, expected)
    # Ids at sampled pixels against the oracle's exact coverage over all triangles.
    g = torch.Generator().manual_seed(1)
    n = 400
    long_idx = torch.randint(0, size, (n,), generator=g)
    short_idx = torch.randint(0, 2, (n,), generator=g)
    rows_s, cols_s = (long_idx, short_idx) if tall else (short_idx, long_idx)
    _, ids = oracle.visible_at_pixels(pos_cpu[0], tri_cpu, *resolution, rows_s, cols_s)
    assert torch.equal(rast[0].cpu()[rows_s, cols_s, 3].long() - 1, ids)
    # The rest of the path on the same image: interpolation, antialiasing and the backward passes.
    attr = torch.rand(pos.shape[1], 3, generator=g).cuda()
    out, out_da = dr.interpolate(attr, rast, tri, rast_db=rast_db, diff_attrs="all")
    image = dr.antialias(out, rast, pos, tri)
    (image.sum() + out_da.sum()).backward()
    assert torch.isfinite(pos.grad).all() and torch.isfinite(image).all()
    assert pos.grad.abs().sum() > 0


@pytest.mark.parametrize("size", [(1, 46342), (1, 65536), (65536, 1)])
def test_level_of_detail_of_very_long_textures(size):
    """Equal to 0.5 (abs 1e-6) and to the oracle (rel 1e-4 / abs 1e-5)."""
    length = max(size)
    tex = (torch.arange(length) % 2).float().view(1, *size, 1)
    centre = (torch.arange(16.0) * 1000 + 0.5) / length
    along_u = size[1] > 1
    uv = torch.full((1, 1, 16, 2), 0.5)
    uv[..., 0 if along_u else 1] = centre
    uv_da = torch.zeros(1, 1, 16, 4)
    uv_da[..., 0 if along_u else 3] = 8.0 / length
    out = dr.texture(tex.cuda(), uv.cuda(), uv_da.cuda(), filter_mode="linear-mipmap-linear")
    torch.testing.assert_close(out.cpu(), torch.full((1, 1, 16, 1), 0.5), atol=1e-6, rtol=0)
    ref = oracle.texture(tex, uv, uv_da, None, None, "linear-mipmap-linear", "wrap")
    torch.testing.assert_close(out.cpu(), ref, atol=1e-5, rtol=1e-4)


def test_rast_db_matches_subpixel_shift(ctx):
    """Moving the triangle by +d in NDC samples it at -d: the central difference of (u, v) over
    a shift of 1e-3 NDC (1/125 pixel at 16 pixels) matches rast_db within 2e-3 + 1e-2 relative
    (float32 rast; the difference quotient of two float32 barycentrics loses about 4 digits)."""
    pos, tri = perspective_triangle()
    pos, tri = pos.cuda(), tri.cuda()
    height, width = 16, 16
    _, rast_db = dr.rasterize(ctx, pos, tri, (height, width))
    eps = 1e-3
    for axis, size, cols in ((0, width, [0, 2]), (1, height, [1, 3])):
        shift = torch.zeros(4, device=CUDA)
        shift[axis] = eps
        plus, _ = dr.rasterize(ctx, pos - shift * pos[..., 3:], tri, (height, width))
        minus, _ = dr.rasterize(ctx, pos + shift * pos[..., 3:], tri, (height, width))
        both = (plus[..., 3] > 0) & (minus[..., 3] > 0)
        assert both.sum() > 50
        fd = (plus[..., :2] - minus[..., :2]) / (2 * eps) * (2 / size)
        torch.testing.assert_close(rast_db[..., cols][both], fd[both], atol=2e-3, rtol=1e-2)


def _coverage(rast):
    return (rast[..., 3:4] > 0).to(rast.dtype)


def _antialias_fd_case(name):
    if name == "constant":
        pos, tri = perspective_triangle()
        return pos, tri, (16, 16), lambda rast, p: _coverage(rast).expand(-1, -1, -1, 3)
    if name == "interpolated":
        pos, tri = perspective_triangle()
        colours = torch.tensor([[1.0, 0.0, 0.2], [0.1, 0.9, 0.3], [0.4, 0.2, 1.0]])

        def color_fn(rast, interp):
            return interp(colours.to(rast.device, rast.dtype), rast)

        return pos, tri, (16, 16), color_fn
    pos = torch.tensor(
        [[[-0.8, -0.7, 0.3, 1.0], [0.9, -0.5, 0.2, 1.2], [-0.2, 0.8, 0.4, 1.1],
          [-0.5, 0.6, -0.2, 1.0], [0.1, -0.9, -0.1, 1.3], [0.8, 0.7, -0.3, 0.9]]])  # fmt: skip
    tri = torch.tensor([[0, 1, 2], [3, 4, 5]], dtype=torch.int32)
    shades = torch.tensor([[0.2, 0.5, 0.9], [0.9, 0.4, 0.1]])

    def color_fn(rast, _):
        ids = rast[..., 3].long()
        s = shades.to(rast.device, rast.dtype)
        return torch.where((ids > 0)[..., None], s[(ids - 1).clamp(min=0)], 0.0)

    return pos, tri, (20, 20), color_fn


@pytest.mark.parametrize("name", ["constant", "interpolated", "overlapping"])
def test_antialias_gradient_matches_finite_differences(ctx, name):
    """d(sum w * antialias(colour)) / d pos on the GPU (float32) against central differences of
    the oracle's float64 image with steps of 1e-6 (x, y and w; z only selects visibility): within
    rel 1e-3 / abs 2e-5 of the largest numeric gradient."""
    pos, tri, resolution, color_fn = _antialias_fd_case(name)
    weights = torch.rand(1, *resolution, 3, generator=torch.Generator().manual_seed(0))

    def gpu_interp(attr, rast):
        return dr.interpolate(attr, rast, tri.cuda())[0]

    def cpu_interp(attr, rast):
        return oracle.interpolate(attr, rast, tri)[0]

    p = pos.cuda().requires_grad_(True)
    rast, _ = dr.rasterize(ctx, p, tri.cuda(), resolution)
    image = dr.antialias(color_fn(rast, gpu_interp), rast, p, tri.cuda())
    (image * weights.cuda()).sum().backward()

    pos64, w64 = pos.double(), weights.double()

    def loss(q):
        r, _ = oracle.rasterize(q, tri, resolution)
        return (oracle.antialias(color_fn(r, cpu_interp), r, q, tri) * w64).sum()

    eps = 1e-6
    numeric = torch.zeros_like(pos64)
    for index in torch.cartesian_prod(*(torch.arange(n) for n in pos.shape)):
        index = tuple(index.tolist())
        if index[-1] == 2:
            continue
        step = torch.zeros_like(pos64)
        step[index] = eps
        numeric[index] = (loss(pos64 + step) - loss(pos64 - step)) / (2 * eps)
    assert numeric.abs().sum() > 0
    cols = [0, 1, 3]
    scale = numeric.abs().max().item()
    torch.testing.assert_close(p.grad.cpu().double()[..., cols], numeric[..., cols], rtol=1e-3,
                               atol=2e-5 * max(1.0, scale))
