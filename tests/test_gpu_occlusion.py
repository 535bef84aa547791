"""The rasterizer's occlusion pass (small triangles facing away set aside, then drawn unless
they lie behind every pixel they touch) gives exactly the keys of a single pass: triangle ids
against the CPU oracle on closed meshes of either winding, through depth peeling and range
mode, and bit-identical rast against the single pass on a 2.6 M-item scene."""

import pytest
import torch

import diffrast_b200 as dr
import oracle
import scenes
from diffrast_b200 import _kernels as K

pytestmark = pytest.mark.gpu
CUDA = "cuda"


@pytest.fixture
def occlusion(monkeypatch):
    monkeypatch.setattr(K, "occlusion_min_items_per_tile", 0.0)


@pytest.fixture(scope="module")
def ctx():
    return dr.RasterizeContext(CUDA)


@pytest.mark.parametrize("flip", [False, True])
def test_closed_mesh_ids_match_oracle(ctx, occlusion, flip):
    sc = scenes.config5_small()
    tri = sc["tri"][:, [0, 2, 1]].contiguous() if flip else sc["tri"]
    rast, _ = dr.rasterize(ctx, sc["pos"].to(CUDA), tri.to(CUDA), sc["resolution"])
    ref, _ = oracle.rasterize(sc["pos"], tri, sc["resolution"])
    assert torch.equal(rast[..., 3].cpu(), ref[..., 3])


def test_peeling_and_ranges_match_oracle(ctx, occlusion):
    sc = scenes.config5_small()
    pos, tri, res = sc["pos"], sc["tri"], sc["resolution"]
    state = None
    with dr.DepthPeeler(ctx, pos.to(CUDA), tri.to(CUDA), res) as peeler:
        for layer in range(3):
            rast, _ = peeler.rasterize_next_layer()
            ref, _, state = oracle.rasterize_layer(pos, tri, res, True, state)
            assert torch.equal(rast[..., 3].cpu(), ref[..., 3]), f"layer {layer}"
    n = tri.shape[0]
    ranges = torch.tensor([[0, n], [n // 3, n // 2], [n // 2, n - n // 2]], dtype=torch.int32)
    rast, _ = dr.rasterize(ctx, pos[0].to(CUDA), tri.to(CUDA), res, ranges=ranges)
    for item, (start, count) in enumerate(ranges.tolist()):
        ref, _ = oracle.rasterize(pos[:1], tri[start : start + count], res)
        ids = ref[0, ..., 3]
        assert torch.equal(rast[item, ..., 3].cpu(), torch.where(ids > 0, ids + start, ids))


def test_occlusion_pass_equals_single_pass_at_scale(ctx, monkeypatch):
    sc = scenes.config5_scene(views=2, resolution=256)
    pos, tri = sc["pos"].to(CUDA), sc["tri"].to(CUDA)
    monkeypatch.setattr(K, "occlusion_min_items_per_tile", float("inf"))
    single, single_db = dr.rasterize(ctx, pos, tri, (256, 256))
    monkeypatch.setattr(K, "occlusion_min_items_per_tile", 0.0)
    two, two_db = dr.rasterize(ctx, pos, tri, (256, 256))
    assert torch.equal(two, single) and torch.equal(two_db, single_db)
