"""The allocation-free edge-adjacency entry point, dr_edge_neighbours_noalloc, called through the
C ABI, against the workspace entry point dr_edge_neighbours on the same index buffers.

It exists for callers that cannot allocate device memory (a plain FFI binding with no device
allocator, or a fixed device-memory budget): its hash table is a fixed 10 MiB device array, so
two calls in a row must each clear what the previous one left there. This file is collected last
so that a failure here does not stop the rest of the suite from running first.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu


def mesh(seed: int, n: int, exact: bool = False) -> torch.Tensor:
    """A grid mesh plus a non-manifold fan and a duplicated triangle, shuffled; with ``exact``,
    topped up with random triangles to exactly ``n``."""
    gen = torch.Generator().manual_seed(seed)
    side = int((n // 2) ** 0.5)
    idx = torch.arange((side + 1) * (side + 1)).view(side + 1, side + 1)
    a, b, c, d = (t.flatten() for t in (idx[:-1, :-1], idx[:-1, 1:], idx[1:, 1:], idx[1:, :-1]))
    tri = torch.cat([torch.stack([a, b, c], -1), torch.stack([a, c, d], -1)])
    extra = torch.tensor([[0, 1, 5000], [1, 0, 5001], [7, 8, 9], [7, 8, 9]])
    tri = torch.cat([tri, extra])
    if exact:
        fill = torch.randint(0, idx.numel(), (n - tri.shape[0], 3), generator=gen)
        tri = torch.cat([tri, fill])
        assert tri.shape[0] == n
    tri = tri[torch.randperm(tri.shape[0], generator=gen)]
    return tri.int().cuda().contiguous()


def call_noalloc(lib, tri, out):
    with torch.cuda.device(tri.device):
        stream = torch.cuda.current_stream().cuda_stream
        status = lib.dr_edge_neighbours_noalloc(tri.data_ptr(), tri.shape[0], out.data_ptr(), stream)
    assert status == 0, lib.dr_status_string(status).decode()


def test_noalloc_matches_workspace_entry_point_on_two_calls_in_a_row():
    from diffrast_b200 import _kernels, _native

    lib = _native.lib()
    assert lib.dr_edge_neighbours_noalloc_max_triangles() == 65536
    for seed, n in ((0, 20000), (1, 6000)):
        tri = mesh(seed, n)
        expected = _kernels.edge_neighbours(tri)
        out = torch.full_like(expected, -7)
        call_noalloc(lib, tri, out)
        torch.cuda.synchronize()
        assert torch.equal(out, expected)
        assert (out >= 0).any() and (out == -1).any()


def test_noalloc_at_its_limit_then_small_allocates_nothing():
    """At exactly the limit the hash table spans the whole array; a smaller call after it must
    ignore the larger table left behind. Neither call may change the device's free memory."""
    from diffrast_b200 import _kernels, _native

    lib = _native.lib()
    limit = lib.dr_edge_neighbours_noalloc_max_triangles()
    big, small = mesh(2, limit, exact=True), mesh(3, 3000)
    expected = [_kernels.edge_neighbours(t) for t in (big, small)]
    outs = [torch.full_like(e, -7) for e in expected]
    call_noalloc(lib, small, outs[1])  # loads the module (and its array) if nothing did yet
    torch.cuda.synchronize()
    outs[1].fill_(-7)
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    for tri, out, exp in zip((big, small), outs, expected):
        call_noalloc(lib, tri, out)
        torch.cuda.synchronize()
        assert torch.equal(out, exp)
    assert torch.cuda.mem_get_info()[0] == free_before


def test_noalloc_refuses_more_than_its_array_holds():
    from diffrast_b200 import _native

    lib = _native.lib()
    tri = torch.zeros(65537, 3, dtype=torch.int32, device="cuda")
    out = torch.empty(65537, 3, dtype=torch.int64, device="cuda")
    status = lib.dr_edge_neighbours_noalloc(tri.data_ptr(), 65537, out.data_ptr(), None)
    assert status == 10004
    assert "65536 triangles" in lib.dr_status_string(status).decode()
