"""CPU check of the oracle's sampled-pixel visibility (``oracle.visible_at_pixels``, used to check
the full-size configurations at sampled pixels) against its whole-image brute force on scenes
with triangles crossing the camera plane, tiny triangles and the spiky config-5 character:
identical ids and depths at every pixel."""

import pytest
import torch

import oracle
import scenes

CASES = {
    "random": lambda: (*scenes.random_mesh(300, torch.Generator().manual_seed(1)), (40, 56)),
    "camera_plane": lambda: (*scenes.random_mesh(400, torch.Generator().manual_seed(3),
                                                 w_range=(-0.6, 2.0)), (48, 40)),
    "tiny": lambda: (*scenes.tiny_mesh(2000, torch.Generator().manual_seed(2), 0.03), (64, 48)),
    "config5_small": lambda: (scenes.config5_small()["pos"], scenes.config5_small()["tri"], (64, 64)),
}


@pytest.mark.parametrize("name", sorted(CASES))
def test_sampled_visibility_equals_brute_force(name):
    pos, tri, (height, width) = CASES[name]()
    depth, ids = oracle.visible_triangles(pos, tri, height, width)
    rows, cols = torch.meshgrid(torch.arange(height), torch.arange(width), indexing="ij")
    rows, cols = rows.flatten(), cols.flatten()
    for view in range(pos.shape[0]):
        d, i = oracle.visible_at_pixels(pos[view], tri, height, width, rows, cols)
        assert torch.equal(i, ids[view].flatten())
        assert torch.equal(d, depth[view].flatten())
    # Scattered pixels in any order give the same answers as the whole image.
    perm = torch.randperm(rows.shape[0], generator=torch.Generator().manual_seed(0))[:200]
    d, i = oracle.visible_at_pixels(pos[0], tri, height, width, rows[perm], cols[perm])
    assert torch.equal(i, ids[0].flatten()[perm])


def test_resolve_at_pixels_matches_whole_image_resolve():
    pos, tri = scenes.random_mesh(200, torch.Generator().manual_seed(6))
    height, width = 32, 24
    _, ids = oracle.visible_triangles(pos, tri, height, width)
    rast, rast_db = oracle.resolve(pos.double(), tri, ids)
    rows, cols = torch.meshgrid(torch.arange(height), torch.arange(width), indexing="ij")
    r, db = oracle.resolve_at_pixels(pos[0].double(), tri, height, width, rows.flatten(),
                                     cols.flatten(), ids[0].flatten())
    assert torch.equal(r, rast[0].reshape(-1, 4)) and torch.equal(db, rast_db[0].reshape(-1, 4))
