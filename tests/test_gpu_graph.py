"""A whole forward + backward step captured into a CUDA graph: no host round trip in any op
(the rasterizer reads its binning counts on the device); replays with new cameras equal eager
runs and the CPU oracle; a visibility pass that outgrows its captured capacity is reported and
poisons its outputs (NaN) instead of being silently wrong.

Tolerances: against eager runs, triangle ids and images exact (same kernels, same inputs), loss
rel 1e-6, gradients rel/abs 1e-4 scaled by the largest value (atomic accumulation order differs
between runs). Against the oracle, as in test_gpu_parity.py: ids bit-exact, image abs 1e-4 /
rel 1e-3, loss abs 1e-5, position gradients 2e-3 and texture gradients 1e-3 (scaled by the
largest gradient).
"""

import pytest
import torch

import diffrast_b200 as dr
import oracle
import scenes

pytestmark = pytest.mark.gpu
CUDA = "cuda"


def close(a, b, tol=1e-4):
    scale = max(1.0, b.abs().max().item())
    torch.testing.assert_close(a, b, atol=tol * scale, rtol=tol)


def make_step(ctx, pos, tex, tri, attr, target, res):
    def step():
        rast, rast_db = dr.rasterize(ctx, pos, tri, res)
        out, out_da = dr.interpolate(attr, rast, tri, rast_db=rast_db, diff_attrs="all")
        color = dr.texture(tex, out[..., 0:2], out_da[..., 0:4], filter_mode="linear-mipmap-linear")
        image, loss = dr.antialias_mse(color, rast, pos, tri, target)
        loss.backward()
        return rast, image, loss

    return step


def oracle_step(pos, tex, tri, attr, target, res):
    """The captured step on the CPU oracle: ids, image, loss and the two gradients."""
    p = pos.detach().cpu().clone().requires_grad_(True)
    t = tex.detach().cpu().clone().requires_grad_(True)
    tri, attr, target = tri.cpu(), attr.cpu(), target.cpu()
    rast, rast_db = oracle.rasterize(p, tri, res)
    out, out_da = oracle.interpolate(attr, rast, tri, rast_db, list(range(attr.shape[-1])))
    color = oracle.texture(t, out[..., 0:2].contiguous(), out_da[..., 0:4].contiguous(), None,
                           None, "linear-mipmap-linear", "wrap")
    image = oracle.antialias(color, rast, p, tri)
    loss = ((image - target) ** 2).mean()
    loss.backward()
    return rast[..., 3], image.detach(), loss.item(), p.grad, t.grad


def capture(step, params):
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(2):
            for p in params:
                p.grad = None
            step()
    torch.cuda.current_stream().wait_stream(side)
    for p in params:
        p.grad = None
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        outputs = step()
    return graph, outputs


def test_captured_step_matches_eager():
    sc = scenes.config5_small()
    ctx = dr.RasterizeContext(CUDA)
    pos = sc["pos"].to(CUDA).requires_grad_(True)
    tex = sc["tex"].to(CUDA).requires_grad_(True)
    tri, attr, target = sc["tri"].to(CUDA), sc["attr"].to(CUDA), sc["target"].to(CUDA)
    step = make_step(ctx, pos, tex, tri, attr, target, sc["resolution"])
    graph, (rast, image, loss) = capture(step, [pos, tex])

    for shift in (0.0, 0.01):  # the captured inputs, then moved vertices copied into them
        with torch.no_grad():
            pos.copy_(sc["pos"].to(CUDA) + shift)
        graph.replay()
        torch.cuda.synchronize()
        assert not ctx.capture_overflowed()
        got = (rast.clone(), image.clone(), loss.clone(), pos.grad.clone(), tex.grad.clone())
        ref_pos = pos.detach().clone().requires_grad_(True)
        ref_tex = tex.detach().clone().requires_grad_(True)
        ref = make_step(ctx, ref_pos, ref_tex, tri, attr, target, sc["resolution"])()
        assert torch.equal(got[0][..., 3], ref[0][..., 3]), "triangle ids"
        assert torch.equal(got[1], ref[1]), "image"
        torch.testing.assert_close(got[2], ref[2], rtol=1e-6, atol=0)
        close(got[3], ref_pos.grad)
        close(got[4], ref_tex.grad)


def test_replays_with_new_cameras_match_the_oracle():
    """The cameras change between replays (new clip positions copied into the captured input);
    every replay is compared with the CPU oracle run on that replay's inputs."""
    sc = scenes.config5_small()
    ctx = dr.RasterizeContext(CUDA)
    res = sc["resolution"]
    pos = sc["pos"].to(CUDA).requires_grad_(True)
    tex = sc["tex"].to(CUDA).requires_grad_(True)
    tri, attr, target = sc["tri"].to(CUDA), sc["attr"].to(CUDA), sc["target"].to(CUDA)
    step = make_step(ctx, pos, tex, tri, attr, target, res)
    graph, (rast, image, loss) = capture(step, [pos, tex])
    world = scenes.icosphere(4)[0]
    world = world * (1 + 0.15 * torch.randn(world.shape[0], 1, generator=torch.Generator().manual_seed(5)))
    gen = torch.Generator().manual_seed(77)
    for _ in range(3):
        mvp = scenes.perspective(45.0) @ scenes.look_at(scenes.orbit_cameras(pos.shape[0], 3.0, gen))
        new_pos = scenes.to_clip(world, mvp)
        with torch.no_grad():
            pos.copy_(new_pos.to(CUDA))
        graph.replay()
        torch.cuda.synchronize()
        assert not ctx.capture_overflowed()
        ids, img, value, g_pos, g_tex = oracle_step(pos, tex, tri, attr, target, res)
        assert torch.equal(rast[..., 3].cpu(), ids), "triangle ids"
        torch.testing.assert_close(image.cpu(), img, atol=1e-4, rtol=1e-3)
        assert abs(loss.item() - value) < 1e-5
        close(pos.grad.cpu(), g_pos, 2e-3)
        close(tex.grad.cpu(), g_tex, 1e-3)


def test_capture_overflow_is_reported_and_poisons_the_outputs():
    from diffrast_b200 import _kernels as K

    # Large overlapping triangles: every one is binned into screen tiles.
    pos, tri = scenes.random_mesh(300, torch.Generator().manual_seed(4), xy_range=0.9)
    ctx = dr.RasterizeContext(CUDA)
    pos, tri = pos.to(CUDA), tri.to(CUDA)
    res = (120, 136)
    eager, eager_db = dr.rasterize(ctx, pos, tri, res)
    covered = eager[..., 3] > 0
    assert covered.any()
    key = (pos.device, 1, tri.shape[0], *res)
    assert key in K._graph_capacity
    full_caps = K._graph_capacity[key]

    def captured_rasterize():
        graph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            with torch.cuda.graph(graph):
                out = dr.rasterize(ctx, pos, tri, res)
        torch.cuda.current_stream().wait_stream(side)
        return graph, out

    # A graph with room for every binned triangle: complete, no overflow, nothing poisoned.
    good, (good_rast, good_db) = captured_rasterize()
    good.replay()
    torch.cuda.synchronize()
    assert not ctx.capture_overflowed()
    assert torch.equal(good_rast, eager) and torch.equal(good_db, eager_db)

    K._graph_capacity[key] = (4, 4)  # far below the binned count
    small, (rast, rast_db) = captured_rasterize()
    small.replay()
    torch.cuda.synchronize()
    # Every covered pixel's barycentrics, depth and derivatives are NaN; ids stay in range.
    ids = rast[..., 3]
    hit = ids > 0
    assert hit.any()
    assert torch.isnan(rast[..., :3][hit]).all() and torch.isnan(rast_db[hit]).all()
    assert (ids <= tri.shape[0]).all() and not torch.isnan(ids).any()
    assert (rast[~hit] == 0).all()
    # The word stays set until checked: the complete graph's replay is poisoned too.
    good.replay()
    torch.cuda.synchronize()
    assert torch.isnan(good_rast[..., :3][good_rast[..., 3] > 0]).all()
    assert ctx.capture_overflowed()
    assert K._graph_capacity[key] == (8, 8)
    assert not ctx.capture_overflowed()
    good.replay()  # once acknowledged, a complete graph gives clean results again
    torch.cuda.synchronize()
    assert torch.equal(good_rast, eager)
    del small, good
    # An eager call afterwards is complete again and restores room for later captures.
    again, _ = dr.rasterize(ctx, pos, tri, res)
    assert torch.equal(again[..., 3], eager[..., 3])
    assert K._graph_capacity[key][0] >= full_caps[0]
