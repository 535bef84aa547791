"""BASELINE configurations at their full stated sizes against the CPU oracle.

Configuration 1 is checked whole: 256 x 256, icosphere-3 under a random rotation, a 256 x 256 x 3
texture sampled with ``linear``, antialiasing and an MSE loss with gradients to the texture and
the positions, end to end on both devices.

Configurations 2 (8 views at 1024 x 1024 of a 65,536-triangle torus knot) and 5 (64 views at
1024 x 1024 of the 1,310,720-triangle displaced icosphere-8: the benchmarked workload) are too
large for the brute-force oracle over whole images, so they are rasterized in full on the GPU and
checked at sampled pixels: a few hundred seeded pixels per view plus every pixel of one 32 x 32
window, with the oracle's exact coverage test evaluated there over every triangle that can reach
the pixel (``oracle.visible_at_pixels``). For configuration 5 the interpolated attributes and the
trilinear texture lookups of the sampled pixels are compared too.

Tolerances: triangle ids and the antialias edge set bit-exact; rast and rast_db within 1e-4
relative (floored at 1) of a float64 recomputation; forward values rel 1e-4 / abs 1e-5 (image
after antialiasing abs 1e-4 / rel 1e-3); loss abs 1e-5; position gradients 2e-3 and texture
gradients 1e-3, scaled by the largest gradient.
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


def sample_pixels(height, width, count, window, seed):
    """``count`` seeded pixels plus every pixel of a 32 x 32 window at ``window`` (row, col)."""
    gen = torch.Generator().manual_seed(seed)
    rows = torch.randint(0, height, (count,), generator=gen)
    cols = torch.randint(0, width, (count,), generator=gen)
    wr, wc = torch.meshgrid(torch.arange(window[0], window[0] + 32),
                            torch.arange(window[1], window[1] + 32), indexing="ij")
    return torch.cat([rows, wr.flatten()]), torch.cat([cols, wc.flatten()])


def check_view_at_samples(pos_view, tri, rast_view, db_view, height, width, rows, cols):
    """Ids at the sampled pixels equal the oracle's; rast / rast_db within 1e-4 of float64."""
    _, ids = oracle.visible_at_pixels(pos_view, tri, height, width, rows, cols)
    ours = rast_view[rows, cols]
    assert torch.equal(ours[:, 3].long() - 1, ids), "triangle ids at sampled pixels"
    exact, exact_db = oracle.resolve_at_pixels(pos_view.double(), tri, height, width, rows, cols, ids)
    for got, truth in ((ours, exact), (db_view[rows, cols], exact_db)):
        err = (got.double() - truth).abs() / truth.abs().clamp_min(1)
        assert err.max() < 1e-4, err.max()
    return ids


def test_config1_exactly_as_stated():
    """The whole configuration on both devices. The oracle's float32 barycentrics can stray from
    the exact values by more than the tolerance where edge functions cancel (one pixel here, 3.7e-4
    off float64), so, as the reference's own backend-parity test does, rast is compared with a
    float64 recomputation, and the oracle's later stages are fed the GPU's rast values (their
    gradients still flow through the oracle's resolve): every stage is compared on the same
    inputs."""
    sc = scenes.config1_scene(seed=0)
    ctx = dr.RasterizeContext(CUDA)
    res = sc["resolution"]
    assert res == (256, 256) and sc["tex"].shape == (1, 256, 256, 3) and sc["tri"].shape[0] == 1280
    tri_c, uv_c, target_c = sc["tri"], sc["uv"], sc["target"]

    pos = sc["pos"].to(CUDA).clone().requires_grad_(True)
    tex = sc["tex"].to(CUDA).clone().requires_grad_(True)
    tri, uv = tri_c.to(CUDA), uv_c.to(CUDA)
    rast, rast_db = dr.rasterize(ctx, pos, tri, res)
    uvp, _ = dr.interpolate(uv, rast, tri)
    color = dr.texture(tex, uvp, filter_mode="linear")
    image = dr.antialias(color, rast, pos, tri)
    loss = torch.nn.functional.mse_loss(image, target_c.to(CUDA))
    loss.backward()
    ours = dict(rast=rast.detach().cpu(), db=rast_db.detach().cpu(), image=image.detach().cpu(),
                loss=loss.item(), g_pos=pos.grad.cpu(), g_tex=tex.grad.cpu(),
                blended=(image != color).detach().cpu())

    p = sc["pos"].clone().requires_grad_(True)
    t = sc["tex"].clone().requires_grad_(True)
    with torch.no_grad():
        _, ids = oracle.visible_triangles(p, tri_c, *res)
    assert torch.equal(ours["rast"][..., 3].long() - 1, ids), "triangle ids"
    assert (ids >= 0).sum() > 10000
    exact, exact_db = oracle.resolve(p.detach().double(), tri_c, ids)
    for got, truth in ((ours["rast"], exact), (ours["db"], exact_db)):
        err = (got.double() - truth).abs() / truth.abs().clamp_min(1)
        assert err.max() < 1e-4, err.max()
    r_ref, _ = oracle.resolve(p, tri_c, ids)
    r_in = ours["rast"] + (r_ref - r_ref.detach())  # GPU values, oracle gradients
    uv_ref, _ = oracle.interpolate(uv_c, r_in, tri_c)
    color_ref = oracle.texture(t, uv_ref, None, None, None, "linear", "wrap")
    image_ref = oracle.antialias(color_ref, r_in, p, tri_c)
    loss_ref = torch.nn.functional.mse_loss(image_ref, target_c)
    loss_ref.backward()
    assert torch.equal(ours["blended"], (image_ref != color_ref).detach()), "antialias edge set"
    assert ours["blended"].any()
    torch.testing.assert_close(ours["image"], image_ref.detach(), atol=1e-4, rtol=1e-3)
    assert abs(ours["loss"] - loss_ref.item()) < 1e-5
    close(ours["g_pos"], p.grad, 2e-3)
    close(ours["g_tex"], t.grad, 1e-3)


def test_config2_full_size_at_sampled_pixels():
    sc = scenes.config2_small(views=8, resolution=1024, segments=512, sides=64)
    assert sc["tri"].shape[0] == 65536 and sc["pos"].shape[:2] == (8, 32768)
    ctx = dr.RasterizeContext(CUDA)
    pos = sc["pos"].to(CUDA).requires_grad_(True)
    tri = sc["tri"].to(CUDA)
    rast, rast_db = dr.rasterize(ctx, pos, tri, sc["resolution"])
    ((rast * sc["g_rast"].to(CUDA)).sum() + (rast_db * sc["g_db"].to(CUDA)).sum()).backward()
    assert torch.isfinite(pos.grad).all() and pos.grad.abs().sum() > 0
    rast, rast_db = rast.detach().cpu(), rast_db.detach().cpu()
    covered = 0
    for view in range(8):
        rows, cols = sample_pixels(1024, 1024, 384, (480 + 4 * view, 496 - 8 * view), seed=20 + view)
        ids = check_view_at_samples(sc["pos"][view], sc["tri"], rast[view], rast_db[view], 1024,
                                    1024, rows, cols)
        covered += int((ids >= 0).sum())
    assert covered > 2000
    # The position gradient of one view against autograd through the oracle's resolve, given the
    # (sampled-checked) ids of the whole view.
    view = 3
    p = sc["pos"][view : view + 1].clone().requires_grad_(True)
    ids = rast[view : view + 1, ..., 3].long() - 1
    r, db = oracle.resolve(p, sc["tri"], ids)
    ((r[..., :3] * sc["g_rast"][view : view + 1, ..., :3]).sum()
     + (db * sc["g_db"][view : view + 1]).sum()).backward()
    p_gpu = sc["pos"][view : view + 1].to(CUDA).requires_grad_(True)
    r_gpu, db_gpu = dr.rasterize(ctx, p_gpu, tri, sc["resolution"])
    ((r_gpu[..., :3] * sc["g_rast"][view : view + 1, ..., :3].to(CUDA)).sum()
     + (db_gpu * sc["g_db"][view : view + 1].to(CUDA)).sum()).backward()
    close(p_gpu.grad, p.grad, 1e-3)


def test_config5_full_size_at_sampled_pixels():
    """The benchmarked workload: 64 views, 1024 x 1024, 1,310,720 triangles, clip positions from
    the world-to-clip kernel as in bench.py. Eight views (every eighth) are sampled."""
    sc = scenes.config5_scene(views=64, resolution=1024, subdivisions=8, tex_size=4096)
    assert sc["tri"].shape[0] == 1310720
    ctx = dr.RasterizeContext(CUDA)
    verts = sc["world"].to(CUDA)
    pos = dr.to_clip(verts, sc["mvp"].to(CUDA))
    tri, attr = sc["tri"].to(CUDA), sc["attr"].to(CUDA)
    tex = sc["tex"].to(CUDA)
    rast, rast_db = dr.rasterize(ctx, pos, tri, sc["resolution"])
    out, out_da = dr.interpolate(attr, rast, tri, rast_db=rast_db, diff_attrs="all")
    color = dr.texture(tex, out[..., 0:2], out_da[..., 0:4], filter_mode="linear-mipmap-linear")
    pos_cpu = pos.cpu()
    torch.testing.assert_close(pos_cpu, sc["pos"], atol=1e-5, rtol=1e-5)  # to_clip vs torch
    rast_c, db_c = rast.cpu(), rast_db.cpu()
    out_c, da_c, color_c = out.cpu(), out_da.cpu(), color.cpu()
    del rast, rast_db, out, out_da, color
    samples = []
    for view in range(0, 64, 8):
        rows, cols = sample_pixels(1024, 1024, 512, (400 + 8 * view, 300 + 4 * view), seed=50 + view)
        ids = check_view_at_samples(pos_cpu[view], sc["tri"], rast_c[view], db_c[view], 1024, 1024,
                                    rows, cols)
        assert (ids >= 0).sum() > 300
        samples.append((view, rows, cols))
    # Interpolation and the trilinear lookup are per pixel: the oracle run on the sampled pixels'
    # rast / rast_db (as a 1 x N image) gives their values.
    views = torch.cat([torch.full_like(r, v) for v, r, _ in samples])
    rows = torch.cat([r for _, r, _ in samples])
    cols = torch.cat([c for _, _, c in samples])
    r_s = rast_c[views, rows, cols][None, None]
    db_s = db_c[views, rows, cols][None, None]
    ref_out, ref_da = oracle.interpolate(sc["attr"], r_s, sc["tri"], db_s, list(range(5)))
    torch.testing.assert_close(out_c[views, rows, cols][None, None], ref_out, atol=1e-5, rtol=1e-4)
    torch.testing.assert_close(da_c[views, rows, cols][None, None], ref_da, atol=1e-5, rtol=1e-4)
    uv = out_c[views, rows, cols][None, None, :, 0:2].contiguous()
    uv_da = da_c[views, rows, cols][None, None, :, 0:4].contiguous()
    ref_color = oracle.texture(sc["tex"], uv, uv_da, None, None, "linear-mipmap-linear", "wrap")
    torch.testing.assert_close(color_c[views, rows, cols][None, None], ref_color, atol=2e-5,
                               rtol=1e-4)
