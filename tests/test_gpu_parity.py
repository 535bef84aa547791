"""Parity of the CUDA kernels with the reference (golden fixtures) and the CPU oracle.

Tolerances (stated per check): triangle ids, coverage, silhouettes and edge adjacency bit-exact;
rast / rast_db within 1e-4 relative (floored at 1) of a float64 recomputation, as the reference's
own backend-parity test does; other forward values rel 1e-4 / abs 1e-5; gradients that are
accumulated with atomics rel/abs 1e-3 (scaled by the largest gradient where they reach large
magnitudes).
"""

import functools

import pytest
import torch

import diffrast_b200 as dr
import oracle
import scenes
from conftest import golden_names, load_golden

pytestmark = pytest.mark.gpu
CUDA = "cuda"


@pytest.fixture(scope="module")
def ctx():
    return dr.RasterizeContext(CUDA)


def fwd_close(a, b, atol=1e-5, rtol=1e-4):
    torch.testing.assert_close(a.cpu(), b.cpu(), atol=atol, rtol=rtol, equal_nan=True)


def grad_close(a, b, tol=1e-3):
    scale = max(1.0, b.abs().max().item()) if b.numel() else 1.0
    torch.testing.assert_close(a.cpu(), b.cpu(), atol=tol * scale, rtol=tol, equal_nan=True)


def check_rast_against_float64(pos, tri, rast, rast_db):
    ids = rast[..., 3].cpu().long() - 1
    exact, exact_db = oracle.resolve(pos.cpu().double(), tri.cpu(), ids)
    for ours, truth in ((rast, exact), (rast_db, exact_db)):
        err = (ours.cpu().double() - truth).abs() / truth.abs().clamp_min(1)
        assert err.max() < 1e-4, err.max()


# ---------------------------------------------------------------------------------------------
# rasterize
# ---------------------------------------------------------------------------------------------


@pytest.mark.parametrize("name", golden_names("raster_"))
def test_rasterize_matches_golden(ctx, name):
    g = load_golden(name)
    res = tuple(g["resolution"].tolist())
    pos, tri = g["pos"].cuda(), g["tri"].cuda()
    p = pos.clone().requires_grad_(True)
    rast, rast_db = dr.rasterize(ctx, p, tri, res)
    assert torch.equal(rast[..., 3].cpu(), g["rast"][..., 3]), "triangle ids must be bit-exact"
    check_rast_against_float64(pos, tri, rast.detach(), rast_db.detach())
    w_rast, w_db = g["w_rast"].cuda(), g["w_db"].cuda()
    ((rast[..., :3] * w_rast[..., :3]).sum() + (rast_db * w_db).sum()).backward()
    grad_close(p.grad, g["grad_pos"])
    with dr.DepthPeeler(ctx, pos, tri, res) as peeler:
        for k in range(g["layer_ids"].shape[0]):
            r, _ = peeler.rasterize_next_layer()
            assert torch.equal(r[..., 3].cpu(), g["layer_ids"][k]), f"layer {k}"


SCENES = {
    "random": lambda: scenes.random_mesh(200, torch.Generator().manual_seed(0), batch=2),
    "crossing_camera": lambda: scenes.random_mesh(60, torch.Generator().manual_seed(2), w_range=(-1.0, 2.0)),
    "clip_and_cull": lambda: scenes.random_mesh(100, torch.Generator().manual_seed(3), z_range=2.0, xy_range=3.0),
    "tiny": lambda: scenes.tiny_mesh(3000, torch.Generator().manual_seed(6), 0.03, batch=2),
    "grid": lambda: scenes.grid_mesh(20, torch.Generator().manual_seed(7), batch=3),
}


@pytest.mark.parametrize("scene", sorted(SCENES))
@pytest.mark.parametrize("res", [(16, 16), (37, 61), (128, 96)])
def test_rasterize_ids_match_oracle(ctx, scene, res):
    pos, tri = SCENES[scene]()
    rast, rast_db = dr.rasterize(ctx, pos.cuda(), tri.cuda(), res)
    ref, _ = oracle.rasterize(pos, tri, res)
    assert torch.equal(rast[..., 3].cpu(), ref[..., 3])
    check_rast_against_float64(pos, tri, rast, rast_db)


def test_rasterize_many_overlapping_large_triangles(ctx):
    # Large overlapping triangles take the binned tile path; many per tile span several work items.
    pos, tri = scenes.random_mesh(600, torch.Generator().manual_seed(4), xy_range=0.9)
    for res in ((16, 16), (200, 180)):
        rast, _ = dr.rasterize(ctx, pos.cuda(), tri.cuda(), res)
        ref, _ = oracle.rasterize(pos, tri, res)
        assert torch.equal(rast[..., 3].cpu(), ref[..., 3])


def test_peeling_every_layer_matches_oracle(ctx):
    gen = torch.Generator().manual_seed(9)
    xy = torch.rand(2, 900, 2, generator=gen) * 3 - 1.5
    z = torch.rand(2, 900, 1, generator=gen) * 2.4 - 1.2
    w = torch.rand(2, 900, 1, generator=gen) * 3 - 1.0
    pos = torch.cat([xy * w, z * w, w], -1)
    tri = torch.arange(900, dtype=torch.int32).view(300, 3)
    for res in ((64, 64), (37, 61)):
        state = None
        with dr.DepthPeeler(ctx, pos.cuda(), tri.cuda(), res) as peeler:
            for layer in range(4):
                rast, _ = peeler.rasterize_next_layer()
                ref, _, state = oracle.rasterize_layer(pos, tri, res, True, state)
                assert torch.equal(rast[..., 3].cpu(), ref[..., 3]), f"layer {layer}"


def test_equal_depth_resolves_to_lower_id(ctx):
    quad = [[-1.0, -1.0, 0.25, 1.0], [1.0, -1.0, 0.25, 1.0], [0.0, 1.0, 0.25, 1.0]]
    pos = torch.tensor([quad * 3], device=CUDA)
    tri = torch.tensor([[6, 7, 8], [0, 1, 2], [3, 4, 5]], dtype=torch.int32, device=CUDA)
    rast, _ = dr.rasterize(ctx, pos, tri, (16, 16))
    covered = rast[..., 3] > 0
    assert covered.any() and (rast[..., 3][covered] == 1).all()


def test_negative_and_zero_depth_ordering(ctx):
    def flat(z):
        return [[-1.0, -1.0, z, 1.0], [3.0, -1.0, z, 1.0], [-1.0, 3.0, z, 1.0]]

    pos = torch.tensor([flat(0.5) + flat(-0.0) + flat(-0.5) + flat(0.0)], device=CUDA)
    tri = torch.arange(12, dtype=torch.int32, device=CUDA).view(4, 3)
    rast, _ = dr.rasterize(ctx, pos, tri, (8, 8))
    assert (rast[..., 3] == 3).all()


def test_empty_culled_and_non_finite(ctx):
    pos = torch.tensor([[[-0.5, -0.5, 0.0, -1.0], [0.5, -0.5, 0.0, -1.0], [0.0, 0.5, 0.0, -1.0]]], device=CUDA)
    tri = torch.tensor([[0, 1, 2]], dtype=torch.int32, device=CUDA)
    for t in (tri, tri[:0]):
        rast, rast_db = dr.rasterize(ctx, pos, t, (16, 16))
        assert (rast == 0).all() and (rast_db == 0).all()
    for value in (float("nan"), float("inf")):
        broken = torch.tensor([[[-0.5, -0.5, 0.0, 1.0], [0.5, -0.5, 0.0, 1.0], [0.0, 0.5, value, 1.0]]], device=CUDA)
        rast, rast_db = dr.rasterize(ctx, broken, tri, (16, 16))
        assert (rast == 0).all() and torch.isfinite(rast_db).all()
    zero = torch.zeros(0, 3, 4, device=CUDA)
    rast, rast_db = dr.rasterize(ctx, zero, tri, (6, 8))
    assert rast.shape == rast_db.shape == (0, 6, 8, 4)


def test_area_tolerance_boundary(ctx):
    # The pixel-(8, 8) centre lies inside a sliver whose area there is 2 * steps / 17 epsilons of
    # its terms: 16 steps is below the two-epsilon tolerance (not drawn), 18 above (drawn).
    eps = torch.finfo(torch.float32).eps
    for steps, drawn in ((4, False), (16, False), (18, True), (64, True)):
        half = 0.5
        centre_x = (8 * 2 + 1) / 16 - 1
        centre_y = (8 * 2 + 1) / 16 - 1
        height = steps * eps * (1 + abs(centre_y)) / 17
        xy = torch.tensor([[centre_x - half, centre_y - height], [centre_x + half, centre_y - height],
                           [centre_x, centre_y + height]], dtype=torch.float64)
        pos = torch.cat([xy.float(), torch.zeros(3, 1), torch.ones(3, 1)], -1)[None]
        tri = torch.tensor([[0, 1, 2]], dtype=torch.int32)
        rast, _ = dr.rasterize(ctx, pos.cuda(), tri.cuda(), (16, 16))
        ref, _ = oracle.rasterize(pos, tri, (16, 16))
        assert torch.equal(rast[..., 3].cpu(), ref[..., 3])


def test_range_mode_matches_instanced_slices(ctx):
    pos, tri = scenes.random_mesh(40, torch.Generator().manual_seed(11))
    ranges = torch.tensor([[0, 10], [5, 20], [30, 10]], dtype=torch.int32)
    rast, _ = dr.rasterize(ctx, pos[0].cuda(), tri.cuda(), (32, 32), ranges=ranges)
    for item, (start, count) in enumerate(ranges.tolist()):
        ref, _ = oracle.rasterize(pos, tri[start : start + count], (32, 32))
        ids = ref[0, ..., 3]
        expected = torch.where(ids > 0, ids + start, ids)
        assert torch.equal(rast[item, ..., 3].cpu(), expected)


def test_range_mode_values_gradients_and_layers(ctx):
    """Range mode in one launch against the reference's per-item loop (diffrast ops.py:482-508):
    overlapping and empty ranges, rast and rast_db values, position gradients summed over the
    items sharing ``pos``, and depth peeling through three layers."""
    pos, tri = scenes.random_mesh(60, torch.Generator().manual_seed(12))
    ranges = torch.tensor([[0, 25], [10, 0], [20, 40], [0, 60], [59, 1]], dtype=torch.int32)
    res = (32, 40)
    gen = torch.Generator().manual_seed(3)
    w_rast = torch.randn(len(ranges), *res, 4, generator=gen)
    w_rast[..., 3] = 0
    w_db = torch.randn(len(ranges), *res, 4, generator=gen)
    p = pos[0].cuda().clone().requires_grad_(True)
    rast, rast_db = dr.rasterize(ctx, p, tri.cuda(), res, ranges=ranges)
    ((rast * w_rast.cuda()).sum() + (rast_db * w_db.cuda()).sum()).backward()
    q = pos[0].clone().requires_grad_(True)
    loss = 0.0
    for item, (start, count) in enumerate(ranges.tolist()):
        ref, ref_db = oracle.rasterize(q[None], tri[start : start + count], res)
        ids = ref[0, ..., 3]
        assert torch.equal(rast[item, ..., 3].cpu(), torch.where(ids > 0, ids + start, ids))
        grad_close(rast[item, ..., :3].detach(), ref[0, ..., :3].detach(), 1e-4)
        grad_close(rast_db[item].detach(), ref_db[0].detach(), 1e-3)
        loss = loss + (ref[0] * w_rast[item]).sum() + (ref_db[0] * w_db[item]).sum()
    loss.backward()
    grad_close(p.grad, q.grad, 1e-3)

    with dr.DepthPeeler(ctx, pos[0].cuda(), tri.cuda(), res, ranges=ranges) as peeler:
        states = [None] * len(ranges)
        for layer in range(3):
            rast, _ = peeler.rasterize_next_layer()
            for item, (start, count) in enumerate(ranges.tolist()):
                ref, _, states[item] = oracle.rasterize_layer(
                    pos, tri[start : start + count], res, True, states[item])
                ids = ref[0, ..., 3]
                expected = torch.where(ids > 0, ids + start, ids)
                assert torch.equal(rast[item, ..., 3].cpu(), expected), f"layer {layer} item {item}"


def test_rasterize_gradients_match_oracle_random(ctx):
    pos, tri = scenes.random_mesh(80, torch.Generator().manual_seed(1), batch=2, w_range=(-1.0, 2.0))
    gen = torch.Generator().manual_seed(0)
    w_rast = torch.randn(2, 40, 56, 4, generator=gen)
    w_db = torch.randn(2, 40, 56, 4, generator=gen)
    for grad_db in (True, False):
        grads = []
        for device in ("cpu", CUDA):
            p = pos.to(device).clone().requires_grad_(True)
            if device == "cpu":
                rast, rast_db = oracle.rasterize(p, tri, (40, 56), grad_db)
            else:
                rast, rast_db = dr.rasterize(ctx, p, tri.cuda(), (40, 56), grad_db=grad_db)
            loss = (rast[..., :3] * w_rast[..., :3].to(device)).sum()
            if rast_db.requires_grad:
                loss = loss + (rast_db * w_db.to(device)).sum()
            loss.backward()
            grads.append(p.grad.cpu())
        grad_close(grads[1], grads[0])


# ---------------------------------------------------------------------------------------------
# interpolate
# ---------------------------------------------------------------------------------------------


@pytest.mark.parametrize("name", golden_names("interp_"))
def test_interpolate_matches_golden(name):
    g = load_golden(name)
    diff = g["diff"].long().tolist()
    a, r, d = (g[k].cuda().clone().requires_grad_(True) for k in ("attr", "rast", "rast_db"))
    out, out_da = dr.interpolate(a, r, g["tri"].cuda(), rast_db=d, diff_attrs=diff or None)
    fwd_close(out, g["out"])
    fwd_close(out_da, g["out_da"])
    ((out * g["g_out"].cuda()).sum() + (out_da * g["g_da"].cuda()).sum()).backward()
    grad_close(a.grad, g["grad_attr"])
    grad_close(r.grad, g["grad_rast"], 1e-4)
    grad_close(d.grad if d.grad is not None else torch.zeros_like(d), g["grad_db"], 1e-4)


@pytest.mark.parametrize("channels", [1, 3, 5, 8, 11])
def test_interpolate_channel_counts_match_oracle(channels):
    """Rows of up to 8 channels are padded to 16 bytes and read with vector loads (1, 3, 5 pad;
    8 does not); more channels take the scalar path. Shared and per-view attributes."""
    pos, tri = scenes.random_mesh(40, torch.Generator().manual_seed(channels), batch=2)
    rast, rast_db = oracle.rasterize(pos, tri, (24, 20))
    gen = torch.Generator().manual_seed(100 + channels)
    for shape in ((pos.shape[1], channels), (2, pos.shape[1], channels)):
        attr = torch.randn(*shape, generator=gen)
        diff = list(range(0, channels, 2))
        g_out = torch.randn(2, 24, 20, channels, generator=gen)
        g_da = torch.randn(2, 24, 20, 2 * len(diff), generator=gen)
        results = []
        for dev in ("cpu", CUDA):
            a = attr.to(dev).clone().requires_grad_(True)
            r = rast.to(dev).clone().requires_grad_(True)
            d = rast_db.to(dev).clone().requires_grad_(True)
            if dev == "cpu":
                out, out_da = oracle.interpolate(a, r, tri, d, diff)
            else:
                out, out_da = dr.interpolate(a, r, tri.to(dev), rast_db=d, diff_attrs=diff)
            ((out * g_out.to(dev)).sum() + (out_da * g_da.to(dev)).sum()).backward()
            results.append((out, out_da, a.grad, r.grad, d.grad))
        ref, ours = results
        fwd_close(ours[0], ref[0])
        fwd_close(ours[1], ref[1])
        for i in (2, 3, 4):
            grad_close(ours[i], ref[i])


def test_interpolate_ids_past_end_are_background():
    rast = torch.zeros(1, 2, 2, 4)
    rast[0, 0, 0] = torch.tensor([0.2, 0.3, 0.0, 1.0])
    rast[0, 0, 1] = torch.tensor([0.2, 0.3, 0.0, 5.0])
    attr = torch.randn(3, 2)
    tri = torch.tensor([[0, 1, 2]], dtype=torch.int32)
    out, _ = dr.interpolate(attr.cuda(), rast.cuda(), tri.cuda())
    ref, _ = oracle.interpolate(attr, rast, tri)
    fwd_close(out, ref)
    assert (out[0, 0, 1] == 0).all()


# ---------------------------------------------------------------------------------------------
# texture
# ---------------------------------------------------------------------------------------------


@pytest.mark.parametrize("name", [n for n in golden_names("tex2d_") if "edge" not in n and "maxmip" not in n])
def test_texture_matches_golden(name):
    g = load_golden(name)
    boundary, mode = name.split("_")[1], name.split("_")[2]
    mip = "mipmap" in mode
    use_bias = bool(g["use_bias"].item())
    t, c, d, bb = (g[k].cuda().clone().requires_grad_(True) for k in ("tex", "uv", "uv_da", "bias"))
    out = dr.texture(t, c, d if mip else None, mip_level_bias=bb if use_bias else None,
                     filter_mode=mode, boundary_mode=boundary)
    fwd_close(out, g["out"], atol=2e-5, rtol=2e-5)
    (out.nan_to_num(0) * g["weights"].cuda()).sum().backward()
    for x, key in ((t, "grad_tex"), (c, "grad_uv"), (d, "grad_uv_da"), (bb, "grad_bias")):
        grad = x.grad if x.grad is not None else torch.zeros_like(x)
        grad_close(grad, g[key])


@pytest.mark.parametrize("boundary", ["wrap", "clamp", "zero"])
def test_texture_non_finite_inputs_match_golden(boundary):
    g = load_golden(f"tex2d_edge_{boundary}")
    out = dr.texture(g["tex"].cuda(), g["uv"].cuda(), g["uv_da"].cuda(),
                     filter_mode="linear-mipmap-linear", boundary_mode=boundary)
    fwd_close(out, g["out"], atol=2e-5, rtol=2e-5)


@pytest.mark.parametrize("level", [0, 2])
def test_texture_max_mip_level_matches_golden(level):
    g = load_golden(f"tex2d_maxmip{level}")
    out = dr.texture(g["tex"].cuda(), g["uv"].cuda(), g["uv_da"].cuda(), max_mip_level=level)
    fwd_close(out, g["out"], atol=2e-5, rtol=2e-5)
    stack = dr.texture_construct_mip(g["tex"].cuda())
    out2 = dr.texture(g["tex"].cuda(), g["uv"].cuda(), g["uv_da"].cuda(), mip=stack, max_mip_level=level)
    fwd_close(out2, g["out"], atol=2e-5, rtol=2e-5)


@pytest.mark.parametrize("name", golden_names("mip_"))
def test_mip_chain_matches_golden(name):
    g = load_golden(name)
    stack = dr.texture_construct_mip(g["tex"].cuda())
    fwd_close(torch.cat([lv.reshape(-1) for lv in stack.levels]), g["levels"])


def test_mip_chain_gradient_matches_oracle():
    gen = torch.Generator().manual_seed(3)
    for h, w in ((37, 50), (16, 9), (1, 7), (64, 64)):
        tex = torch.randn(2, h, w, 3, generator=gen)
        weights = [torch.randn_like(lv) for lv in oracle.mip_chain(tex)[1:]]
        grads = []
        for device in ("cpu", CUDA):
            t = tex.to(device).clone().requires_grad_(True)
            levels = oracle.mip_chain(t)[1:] if device == "cpu" else dr.texture_construct_mip(t).levels
            sum((lv * wt.to(device)).sum() for lv, wt in zip(levels, weights)).backward()
            grads.append(t.grad.cpu())
        grad_close(grads[1], grads[0], 1e-4)


def test_whole_mip_chain_equals_one_step_at_a_time():
    """dr_mip_build (runs of even halvings several levels per launch) and dr_mip_build_bwd (the
    adjoint chain in one call) against one dr_mip_downsample / dr_mip_downsample_bwd call per
    level: bit-identical, for power-of-two, partly even and odd sizes, 1 to 5 channels, several
    images, in place and into an unpadded output."""
    from diffrast_b200 import _kernels as K

    gen = torch.Generator().manual_seed(17)
    shapes = [(1, 256, 256, 3), (2, 128, 64, 1), (1, 96, 40, 4), (3, 48, 48, 5), (1, 1, 64, 2),
              (12, 32, 32, 3), (1, 4096, 8, 3)]
    for shape in shapes:
        tex = torch.rand(shape, generator=gen).cuda()
        count = 0
        h, w = shape[1], shape[2]
        while h > 1 or w > 1:
            h, w = (h + 1) // 2, (w + 1) // 2
            count += 1
        whole = K.mip_build(tex, count)
        steps, level = [], tex
        for _ in range(count):
            level = K.mip_down(level)
            steps.append(level)
        for a, b in zip(whole, steps):
            assert torch.equal(a, b), shape
        stride = 4 if shape[-1] == 3 else shape[-1]
        grads = [torch.randn((*lv.shape[:-1], stride), generator=gen).cuda()
                 for lv in [tex, *steps]]
        for unpadded in (False, True):
            ref = [g.clone() for g in grads]
            out_ref = torch.empty(shape, device=CUDA) if unpadded else None
            for level in range(len(ref) - 2, -1, -1):
                K.mip_down_bwd(ref[level + 1], ref[level], out_ref if level == 0 else None)
            got = [g.clone() for g in grads]
            out = torch.empty(shape, device=CUDA) if unpadded else None
            K.mip_build_bwd(got, out)
            if unpadded:
                assert torch.equal(out, out_ref), shape
                assert torch.equal(got[0], grads[0]), shape  # left unchanged
            else:
                assert torch.equal(got[0], ref[0]), shape


@pytest.mark.parametrize("name", golden_names("cube_"))
def test_cube_texture_matches_golden(name):
    g = load_golden(name)
    mode = name[len("cube_"):]
    mip = "mipmap" in mode
    t, d, dd = (g[k].cuda().clone().requires_grad_(True) for k in ("tex", "dirs", "dirs_da"))
    out = dr.texture(t, d, dd if mip else None, filter_mode=mode, boundary_mode="cube")
    fwd_close(out, g["out"], atol=2e-5, rtol=2e-5)
    (out * g["weights"].cuda()).sum().backward()
    for x, key in ((t, "grad_tex"), (d, "grad_dirs"), (dd, "grad_dirs_da")):
        grad = x.grad if x.grad is not None else torch.zeros_like(x)
        grad_close(grad, g[key])


def test_texture_shared_texels_gradients_match_oracle():
    gen = torch.Generator().manual_seed(5)
    tex = torch.randn(2, 37, 50, 3, generator=gen)
    uv_da = (torch.rand(2, 20, 24, 4, generator=gen) * 0.2 - 0.1)
    base_uv = torch.rand(2, 20, 24, 2, generator=gen) * 1.6 - 0.3
    for pattern in ("constant", "magnified", "mixed"):
        uv = base_uv.clone()
        if pattern == "constant":
            uv = torch.full_like(uv, 0.3)
        elif pattern == "magnified":
            uv = uv / 16 + 0.4
        else:
            uv[:, ::2] = 0.0
        for mode in ("nearest", "linear", "linear-mipmap-nearest", "linear-mipmap-linear"):
            mip = "mipmap" in mode
            grads = []
            for device in ("cpu", CUDA):
                t = tex.to(device).clone().requires_grad_(True)
                if device == "cpu":
                    out = oracle.texture(t, uv, uv_da if mip else None, None, None, mode, "clamp")
                else:
                    out = dr.texture(t, uv.cuda(), uv_da.cuda() if mip else None, filter_mode=mode, boundary_mode="clamp")
                out.sum().backward()
                grads.append(t.grad.cpu())
            grad_close(grads[1], grads[0])


# ---------------------------------------------------------------------------------------------
# antialias
# ---------------------------------------------------------------------------------------------


@pytest.mark.parametrize("name", golden_names("aa_"))
def test_antialias_matches_golden(name):
    g = load_golden(name)
    tri = g["tri"].cuda()
    nb = dr.antialias_construct_topology_hash(tri).neighbours(tri)
    assert torch.equal(nb.cpu(), g["neighbours"]), "edge adjacency must be bit-exact"
    from diffrast_b200 import _kernels as K

    pos3 = g["pos"].cuda() if g["pos"].ndim == 3 else g["pos"].cuda()[None]
    assert torch.equal(K.silhouette_edges(pos3, tri, nb).cpu(), g["silhouette"]), "silhouettes"
    c = g["color"].cuda().clone().requires_grad_(True)
    p = g["pos"].cuda().clone().requires_grad_(True)
    out = dr.antialias(c, g["rast"].cuda(), p, tri, pos_gradient_boost=float(g["boost"]))
    fwd_close(out, g["out"])
    (out * g["weights"].cuda()).sum().backward()
    grad_close(c.grad, g["grad_color"], 1e-5)
    grad_close(p.grad, g["grad_pos"])


def test_antialias_edge_set_matches_oracle_random():
    for seed, mesh in ((0, {}), (1, {"w_range": (-1.0, 2.0)}), (2, {"z_range": 2.0, "xy_range": 3.0})):
        pos, tri = scenes.random_mesh(60, torch.Generator().manual_seed(seed), batch=2, **mesh)
        rast, _ = oracle.rasterize(pos, tri, (48, 64))
        color = torch.rand(2, 48, 64, 3, generator=torch.Generator().manual_seed(seed + 10))
        ref = oracle.antialias(color, rast, pos, tri)
        out = dr.antialias(color.cuda(), rast.cuda(), pos.cuda(), tri.cuda())
        # Same set of blended pixels, same values.
        assert torch.equal((out.cpu() != color), (ref != color))
        fwd_close(out, ref)


def test_antialias_recorded_pairs_match_recomputed_pairs():
    """The backward pass from the forward pass's pair records equals the one that repeats the
    edge tests (the C ABI offers both)."""
    from diffrast_b200 import _kernels as K

    for seed in (0, 1):
        pos, tri = scenes.random_mesh(80, torch.Generator().manual_seed(seed), batch=2)
        rast, _ = oracle.rasterize(pos, tri, (40, 56))
        gen = torch.Generator().manual_seed(seed + 20)
        color = torch.rand(2, 40, 56, 3, generator=gen).cuda()
        grad_out = torch.randn(2, 40, 56, 3, generator=gen).cuda()
        pos, tri, rast = pos.cuda(), tri.cuda(), rast.cuda()
        opp = dr.antialias_construct_topology_hash(tri).opposite(tri)
        out, pairs = K.antialias_fwd(color, rast, pos, tri, opp, record_pairs=True)
        out_plain, none = K.antialias_fwd(color, rast, pos, tri, opp)
        assert none is None and torch.equal(out, out_plain)
        gc_rec, gp_rec = K.antialias_bwd(color, rast, pos, tri, opp, grad_out, 1.0, pairs)
        gc, gp = K.antialias_bwd(color, rast, pos, tri, opp, grad_out, 1.0)
        torch.testing.assert_close(gc_rec, gc, rtol=1e-6, atol=1e-7)
        # Position gradients are sums of atomically added terms: only their order may differ
        # (the atomic-gradient tolerance of this file).
        grad_close(gp_rec, gp)
        assert (gp != 0).any()


def test_straight_edge_coverage_is_exact(ctx):
    edge = 0.3
    pos = torch.tensor([[[-2.0, -2.0, 0.0, 1.0], [edge, -2.0, 0.0, 1.0], [edge, 2.0, 0.0, 1.0],
                         [-2.0, 2.0, 0.0, 1.0]]], device=CUDA)
    tri = torch.tensor([[0, 1, 2], [0, 2, 3]], dtype=torch.int32, device=CUDA)
    rast, _ = dr.rasterize(ctx, pos, tri, (16, 24))
    out = dr.antialias((rast[..., 3:] > 0).float(), rast, pos, tri)
    torch.testing.assert_close(out.sum().cpu(), torch.tensor(16 * (edge + 1) * 24 / 2))


def test_edge_neighbours_match_golden():
    g = load_golden("topology")
    for key, nkey in (("tri", "neighbours"), ("tri_fan", "neighbours_fan")):
        tri = g[key].cuda()
        topo = dr.antialias_construct_topology_hash(tri)
        nb = topo.neighbours(tri)
        assert torch.equal(nb.cpu(), g[nkey])
        # The kernels' form: tri[neighbours] (the vertex across each edge), -1 where unshared.
        expected = torch.where(g[nkey] >= 0, g[key].reshape(-1)[g[nkey].clamp_min(0)], -1)
        assert torch.equal(topo.opposite(tri).cpu(), expected.int())


# ---------------------------------------------------------------------------------------------
# full pipeline
# ---------------------------------------------------------------------------------------------


def test_texture_of_interpolated_slices_routes_gradients(ctx):
    """uv = out[..., 0:2] and uv_da = out_da[..., 0:4] of interpolate: the lookup hands its compact
    coordinate gradients back to the interpolation (no whole gradient images); the result equals
    passing copies."""
    sc = scenes.config1_scene(seed=2)
    pos, tri = sc["pos"].cuda(), sc["tri"].cuda()
    gen = torch.Generator().manual_seed(5)
    attr = torch.cat([sc["uv"], torch.rand(sc["uv"].shape[0], 3, generator=gen)], -1).cuda()
    tex = torch.rand(1, 64, 64, 3, generator=gen).cuda()
    weights = torch.randn(1, 48, 48, 3, generator=gen).cuda()
    rast, rast_db = dr.rasterize(ctx, pos, tri, (48, 48))
    for mode, mip in (("linear-mipmap-linear", None), ("linear-mipmap-linear", "stack"),
                      ("linear", None)):
        results = []
        for copy in (False, True):
            a = attr.clone().requires_grad_(True)
            t = tex.clone().requires_grad_(True)
            out, out_da = dr.interpolate(a, rast, tri, rast_db=rast_db, diff_attrs="all")
            uv, uv_da = out[..., 0:2], out_da[..., 0:4]
            if copy:
                uv, uv_da = uv.clone(), uv_da.clone()
            stack = dr.texture_construct_mip(t) if mip else None
            color = dr.texture(t, uv, uv_da, mip=stack, filter_mode=mode)
            grads = torch.autograd.grad((color * weights).sum(), [a, t])
            results.append((color, *grads))
        for ours, ref in zip(results[0], results[1]):
            grad_close(ours, ref, 1e-5)


def test_coordinate_port_with_other_consumers_and_retained_graphs(ctx):
    """The hand-over of lookup gradients to interpolate (a zero-size port output) against copies
    of the slices, where it is hardest: other ops also use out and out_da, two lookups read
    different slices of one interpolation, a lookup reads uv without uv_da (and one reads uv_da
    that is not interpolate's), and a retained graph is differentiated twice, first only with
    respect to the texture (so the interpolation's backward does not run that time)."""
    sc = scenes.config1_scene(seed=3)
    pos, tri = sc["pos"].cuda(), sc["tri"].cuda()
    gen = torch.Generator().manual_seed(11)
    attr = torch.cat([sc["uv"], torch.rand(sc["uv"].shape[0], 4, generator=gen)], -1).cuda()
    tex = torch.rand(1, 32, 32, 3, generator=gen).cuda()
    w1, w2, w3 = (torch.randn(1, 40, 40, k, generator=gen).cuda() for k in (3, 3, 6))
    rast, rast_db = dr.rasterize(ctx, pos, tri, (40, 40))
    foreign_da = torch.rand(1, 40, 40, 4, generator=gen).cuda() * 0.01

    def run(copy: bool, case: str):
        a = attr.clone().requires_grad_(True)
        t = tex.clone().requires_grad_(True)
        out, out_da = dr.interpolate(a, rast, tri, rast_db=rast_db, diff_attrs="all")

        def s(x):
            return x.clone() if copy else x

        mode = "linear-mipmap-linear"
        if case == "other_consumers":
            color = dr.texture(t, s(out[..., 0:2]), s(out_da[..., 0:4]), filter_mode=mode)
            loss = (color * w1).sum() + (out[..., 2:6] ** 2).sum() + (out_da * w3[..., :1]).sum()
        elif case == "two_lookups":
            c1 = dr.texture(t, s(out[..., 0:2]), s(out_da[..., 0:4]), filter_mode=mode)
            c2 = dr.texture(t, s(out[..., 2:4]), s(out_da[..., 4:8]), filter_mode=mode)
            c3 = dr.texture(t, s(out[..., 0:2]), s(out_da[..., 0:4]), filter_mode="linear")
            loss = (c1 * w1).sum() + (c2 * w2).sum() + (c3 * w1).sum()
        elif case == "uv_only":
            c1 = dr.texture(t, s(out[..., 1:3]), filter_mode="linear")
            c2 = dr.texture(t, s(out[..., 0:2]), foreign_da, filter_mode=mode)
            loss = (c1 * w1).sum() + (c2 * w2).sum()
        else:  # retained graph
            color = dr.texture(t, s(out[..., 0:2]), s(out_da[..., 0:4]), filter_mode=mode)
            loss = (color * w1).sum()
            first = torch.autograd.grad(loss, [t], retain_graph=True)[0]
            return (first, *torch.autograd.grad(loss, [a, t]))
        return torch.autograd.grad(loss, [a, t])

    for case in ("other_consumers", "two_lookups", "uv_only", "retained"):
        ours, ref = run(False, case), run(True, case)
        for x, y in zip(ours, ref):
            grad_close(x, y, 1e-5)


def test_lookup_with_fused_interpolation_backward(ctx):
    """A 2D lookup of interpolated channels whose attributes need no gradient runs the
    interpolation's backward pass for its coordinates inside its own (dr_texture_bwd_interp) and
    hands over gradients of rast and rast_db. Against the separate passes (fusion off: compact
    coordinate gradients, then the interpolation backward kernel) the gradients are bit-identical
    (rast's and rast_db's) where the lookup is their only source (also when it reads the
    interpolation's outputs whole rather than channel slices of them); against copies of the slices (no hand-over at all)
    they agree within float32 rounding, also where the chained gradients are combined with other
    consumers' or with a second lookup's, where attributes need a gradient (no fusion), and in a
    retained graph differentiated twice (the second pass hands over compact gradients)."""
    from diffrast_b200 import _functions as F

    sc = scenes.config5_small(views=2)
    gen = torch.Generator().manual_seed(31)
    pos, tri = sc["pos"].cuda(), sc["tri"].cuda()
    attr = torch.cat([sc["attr"], torch.rand(sc["attr"].shape[0], 3, generator=gen)], -1).cuda()
    per_view = torch.stack([attr, attr.flip(-1)]).contiguous()  # [views, V, C]: attr_batch 2
    tex = torch.rand(1, 32, 32, 3, generator=gen).cuda()
    w1, w2 = (torch.randn(2, 64, 64, 3, generator=gen).cuda() for _ in range(2))
    w_da = torch.randn(2, 64, 64, 16, generator=gen).cuda()
    rast0, db0 = (x.detach() for x in dr.rasterize(ctx, pos, tri, (64, 64)))

    def run(how: str, case: str):
        F.FUSE_INTERPOLATION_BACKWARD = how != "separate"
        F.DEFER_CHAINED_BACKWARD = how == "deferred"
        try:
            r = rast0.clone().requires_grad_(True)
            d = db0.clone().requires_grad_(True)
            t = tex.clone().requires_grad_(True)
            a = (per_view if case == "attr_batch" else attr).clone()
            if case == "attr_grad":
                a.requires_grad_(True)
            out, out_da = dr.interpolate(a, r, tri, rast_db=d, diff_attrs="all")

            def s(x):
                return x.clone() if how == "copy" else x

            mode = "linear-mipmap-linear"
            uv, uv_da = s(out[..., 0:2]), s(out_da[..., 0:4])
            if case == "whole":  # interpolate's outputs themselves, as the reference's benchmark
                out, out_da = dr.interpolate(a[..., 0:2].contiguous(), r, tri, rast_db=d,
                                             diff_attrs="all")
                uv, uv_da = s(out), s(out_da)
            if case in ("chain", "whole", "attr_batch", "attr_grad", "retained"):
                loss = (dr.texture(t, uv, uv_da, filter_mode=mode) * w1).sum()
            elif case == "stack":
                color = dr.texture(t, uv, uv_da, mip=dr.texture_construct_mip(t), filter_mode=mode)
                loss = (color * w1).sum()
            elif case == "linear":
                loss = (dr.texture(t, uv, filter_mode="linear") * w1).sum()
            elif case == "mip_nearest":
                loss = (dr.texture(t, uv, uv_da, filter_mode="linear-mipmap-nearest") * w1).sum()
            elif case == "offset":
                color = dr.texture(t, s(out[..., 5:7]), s(out_da[..., 10:14]), filter_mode=mode)
                loss = (color * w1).sum()
            elif case == "other_consumers":
                loss = (dr.texture(t, uv, uv_da, filter_mode=mode) * w1).sum() + \
                    (out[..., 2:] ** 2).sum() + (out_da * w_da).sum()
            else:  # two lookups of one interpolation: the second hands over compact gradients
                c2 = dr.texture(t, s(out[..., 3:5]), s(out_da[..., 6:10]), filter_mode=mode)
                loss = (dr.texture(t, uv, uv_da, filter_mode=mode) * w1).sum() + (c2 * w2).sum()
            leaves = [r, d, t] + ([a] if case == "attr_grad" else [])
            grad = functools.partial(torch.autograd.grad, allow_unused=True, materialize_grads=True)
            if case == "retained":
                first = grad(loss, leaves, retain_graph=True)
                return (*first, *grad(loss, leaves))
            return grad(loss, leaves)
        finally:
            F.FUSE_INTERPOLATION_BACKWARD = True
            F.DEFER_CHAINED_BACKWARD = False

    exact = ("chain", "whole", "stack", "linear", "mip_nearest", "offset", "attr_batch")
    for case in exact + ("other_consumers", "two_lookups", "attr_grad", "retained"):
        fused, deferred, separate, copied = (run(how, case)
                                             for how in ("fused", "deferred", "separate", "copy"))
        for i, (x, d, y, z) in enumerate(zip(fused, deferred, separate, copied)):
            if case in exact and i < 2:  # rast, rast_db (the texel gradients use atomics)
                assert torch.equal(x, y) and torch.equal(d, y), case
            grad_close(x, z, 1e-5)
            grad_close(d, z, 1e-5)
        assert fused[0].abs().sum() > 0, case
        if case not in ("linear", "mip_nearest"):
            assert fused[1].abs().sum() > 0, case


def test_lookup_with_fused_rasterizer_backward(ctx):
    """A lookup of coordinates interpolated from rasterize's own rast also runs the rasterizer's
    backward pass in its own (dr_texture_bwd_resolve), adding the position gradient to the
    buffer the rasterizer's backward pass collects. Position and texture gradients against the
    interpolation-only fusion, the separate passes and copies (no hand-over at all), within
    float32 rounding (the position gradient is accumulated with atomics), and with the chained
    part deferred to the interpolation's backward pass (as on several GPUs): with the fused-loss
    antialias (whose position gradient is the buffer), without antialias, with another gradient
    reaching rast (its depth), without a differentiable rast_db, with a bilinear lookup (no
    rast_db gradient from it), and through a retained graph differentiated twice."""
    from diffrast_b200 import _functions as F

    sc = scenes.config5_small(views=2)
    gen = torch.Generator().manual_seed(41)
    pos0, tri = sc["pos"].cuda(), sc["tri"].cuda()
    attr = sc["attr"].cuda()
    tex0 = torch.rand(1, 32, 32, 3, generator=gen).cuda()
    target = sc["target"].cuda()
    w = torch.randn(2, 64, 64, 3, generator=gen).cuda()

    def run(how: str, case: str):
        F.FUSE_INTERPOLATION_BACKWARD = how in ("fused", "deferred", "interp_only")
        F.FUSE_RASTERIZE_BACKWARD = how in ("fused", "deferred")
        F.DEFER_CHAINED_BACKWARD = how == "deferred"
        try:
            pos = pos0.clone().requires_grad_(True)
            tex = tex0.clone().requires_grad_(True)
            rast, rast_db = dr.rasterize(ctx, pos, tri, (64, 64), grad_db=case != "no_db")
            r_in = rast.clone() if how == "copy" else rast
            out, out_da = dr.interpolate(attr, r_in, tri, rast_db=rast_db, diff_attrs="all")
            uv, uv_da = out[..., 0:2], out_da[..., 0:4]
            if how == "copy":
                uv, uv_da = uv.clone(), uv_da.clone()
            mode = "linear" if case == "linear" else "linear-mipmap-linear"
            color = dr.texture(tex, uv, uv_da if mode != "linear" else None, filter_mode=mode)
            if case in ("aa_mse", "retained"):
                _, loss = dr.antialias_mse(color, rast, pos, tri, target)
            else:
                loss = (color * w).sum()
            if case == "depth_too":
                loss = loss + (rast[..., 2] ** 2).sum()
            grad = functools.partial(torch.autograd.grad, allow_unused=True, materialize_grads=True)
            if case == "retained":
                first = grad(loss, [pos, tex], retain_graph=True)
                return (*first, *grad(loss, [pos, tex]))
            return grad(loss, [pos, tex])
        finally:
            F.FUSE_INTERPOLATION_BACKWARD = F.FUSE_RASTERIZE_BACKWARD = True
            F.DEFER_CHAINED_BACKWARD = False

    hows = ("fused", "deferred", "interp_only", "separate", "copy")
    for case in ("aa_mse", "plain", "depth_too", "no_db", "linear", "retained"):
        results = {how: run(how, case) for how in hows}
        for how in hows[1:]:
            for x, y in zip(results["fused"], results[how]):
                grad_close(x, y, 1e-5)
        assert results["fused"][0].abs().sum() > 0, case


def test_position_port_matches_separate_gradients(ctx):
    """Antialias hands its position gradient to the rasterizer's backward pass when it gets the
    rast and the very pos tensor of one rasterize call; against a copy of pos (no hand-over,
    autograd adds the two gradients): plain and fused-loss antialias, two antialias passes over one
    rast, rast_db and interpolation in the loss or not, and a retained graph differentiated first
    with respect to the colour only."""
    sc = scenes.config5_small(views=2)
    gen = torch.Generator().manual_seed(21)
    pos0, tri = sc["pos"].cuda(), sc["tri"].cuda()
    attr = sc["attr"].cuda()
    color0 = torch.rand(2, 64, 64, 3, generator=gen).cuda()
    target = sc["target"].cuda()
    w = torch.randn(2, 64, 64, 3, generator=gen).cuda()

    def run(copy: bool, case: str):
        pos = pos0.clone().requires_grad_(True)
        color = color0.clone().requires_grad_(True)
        rast, rast_db = dr.rasterize(ctx, pos, tri, (64, 64))
        p_aa = pos.clone() if copy else pos
        if case == "plain":
            loss = (dr.antialias(color, rast, p_aa, tri) * w).sum()
        elif case == "fused":
            out, _ = dr.interpolate(attr, rast, tri, rast_db=rast_db, diff_attrs="all")
            _, loss = dr.antialias_mse(color * out[..., 2:5], rast, p_aa, tri, target)
        elif case == "twice":
            loss = (dr.antialias(color, rast, p_aa, tri) * w).sum() + \
                (dr.antialias(color * 2, rast, p_aa, tri, pos_gradient_boost=3.0) ** 2).sum()
        else:  # retained graph, antialias only (no gradient reaches rast itself)
            loss = (dr.antialias(color, rast, p_aa, tri) * w).sum()
            first = torch.autograd.grad(loss, [color], retain_graph=True)[0]
            return (first, *torch.autograd.grad(loss, [pos, color]))
        return torch.autograd.grad(loss, [pos, color])

    for case in ("plain", "fused", "twice", "retained"):
        ours, ref = run(False, case), run(True, case)
        for x, y in zip(ours, ref):
            grad_close(x, y, 1e-5)
        assert ours[-2].abs().sum() > 0


def test_config1_pipeline_matches_oracle(ctx):
    sc = scenes.config1_scene(seed=0)
    res = (64, 64)
    tex_small = sc["tex"][:, :64, :64].contiguous()
    target = torch.rand(1, 64, 64, 3, generator=torch.Generator().manual_seed(1))

    def run(device):
        pos = sc["pos"].to(device).clone().requires_grad_(True)
        tex = tex_small.to(device).clone().requires_grad_(True)
        tri, uv = sc["tri"].to(device), sc["uv"].to(device)
        if device == "cpu":
            rast, rast_db = oracle.rasterize(pos, tri, res)
            uvp, uv_da = oracle.interpolate(uv, rast, tri, rast_db, [0, 1])
            color = oracle.texture(tex, uvp, uv_da, None, None, "linear-mipmap-linear", "wrap")
            out = oracle.antialias(color, rast, pos, tri)
        else:
            rast, rast_db = dr.rasterize(ctx, pos, tri, res)
            uvp, uv_da = dr.interpolate(uv, rast, tri, rast_db=rast_db, diff_attrs="all")
            color = dr.texture(tex, uvp, uv_da, filter_mode="linear-mipmap-linear")
            out = dr.antialias(color, rast, pos, tri)
        loss = ((out - target.to(device)) ** 2).mean()
        loss.backward()
        return out.detach().cpu(), loss.item(), pos.grad.cpu(), tex.grad.cpu()

    ref, ours = run("cpu"), run(CUDA)
    fwd_close(ours[0], ref[0], atol=1e-4, rtol=1e-3)
    assert abs(ours[1] - ref[1]) < 1e-5
    grad_close(ours[2], ref[2], 2e-3)
    grad_close(ours[3], ref[3], 1e-3)


def test_second_order_gradients_are_refused(ctx):
    """Every op's backward is first-order only, like the reference's guard
    (diffrast backends/_autograd.py:11-35): asking it to build a graph raises."""
    pos, tri = scenes.random_mesh(20, torch.Generator().manual_seed(5))
    pos = pos.cuda().requires_grad_(True)
    tri = tri.cuda()
    tex = torch.rand(1, 16, 16, 3, device=CUDA, requires_grad=True)
    world = torch.rand(9, 3, device=CUDA, requires_grad=True)
    mats = torch.eye(4, device=CUDA)[None].repeat(2, 1, 1)
    rast = dr.rasterize(ctx, pos.detach(), tri, (16, 16))[0]
    cases = [
        lambda: dr.rasterize(ctx, pos, tri, (16, 16))[0][..., :3],
        lambda: dr.interpolate(pos[0, :, :3].contiguous(), rast, tri)[0],
        lambda: dr.texture(tex, torch.rand(1, 8, 8, 2, device=CUDA)),
        lambda: dr.antialias(torch.rand(1, 16, 16, 3, device=CUDA, requires_grad=True), rast, pos,
                             tri),
        lambda: dr.to_clip(world, mats),
    ]
    for make in cases:
        out = make()
        with pytest.raises(RuntimeError, match="no second-order gradients"):
            torch.autograd.grad(out.sum(), [pos, tex, world], create_graph=True, allow_unused=True)
