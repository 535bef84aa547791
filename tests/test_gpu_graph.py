"""A whole forward + backward step captured into a CUDA graph: no host round trip in any op
(the rasterizer reads its binning counts on the device), replays equal to eager runs, and a
visibility pass that outgrows its captured capacity is reported instead of silently wrong.

Tolerances: triangle ids and images exact (same kernels, same inputs); loss rel 1e-6; gradients
rel/abs 1e-4 scaled by the largest value (atomic accumulation order differs between runs).
"""

import pytest
import torch

import diffrast_b200 as dr
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


def test_capture_overflow_is_reported():
    from diffrast_b200 import _kernels as K

    # Large overlapping triangles: every one is binned into screen tiles.
    pos, tri = scenes.random_mesh(300, torch.Generator().manual_seed(4), xy_range=0.9)
    ctx = dr.RasterizeContext(CUDA)
    pos, tri = pos.to(CUDA), tri.to(CUDA)
    res = (120, 136)
    eager, _ = dr.rasterize(ctx, pos, tri, res)
    key = (pos.device, 1, tri.shape[0], *res)
    assert key in K._graph_capacity
    K._graph_capacity[key] = (4, 4)  # far below the binned count
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        with torch.cuda.graph(graph):
            rast, _ = dr.rasterize(ctx, pos, tri, res)
    torch.cuda.current_stream().wait_stream(side)
    graph.replay()
    torch.cuda.synchronize()
    assert ctx.capture_overflowed()
    assert K._graph_capacity[key] == (8, 8)
    assert not ctx.capture_overflowed()
    del graph
    # An eager call afterwards is complete again and restores room for later captures.
    again, _ = dr.rasterize(ctx, pos, tri, res)
    assert torch.equal(again[..., 3], eager[..., 3])
    assert K._graph_capacity[key][0] > 8
