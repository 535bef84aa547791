"""Seeded synthetic scenes shared by the golden-fixture generator, the tests and the bench.

All generators run on the CPU with ``torch.Generator`` seeds, so the same call gives the same
tensors here and on a GPU box.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def random_mesh(num_tri, gen, batch=1, z_range=0.9, w_range=(1.0, 2.0), xy_range=1.2):
    """Unconnected triangles with random clip-space corners; ``w`` may cross the camera plane."""
    n = 3 * num_tri
    xy = (torch.rand(batch, n, 2, generator=gen) * 2 - 1) * xy_range
    z = (torch.rand(batch, n, 1, generator=gen) * 2 - 1) * z_range
    w = torch.rand(batch, n, 1, generator=gen) * (w_range[1] - w_range[0]) + w_range[0]
    pos = torch.cat([xy * w, z * w, w], -1)
    tri = torch.arange(n, dtype=torch.int32).view(num_tri, 3)
    return pos, tri


def tiny_mesh(num_tri, gen, size, batch=1):
    """Triangles about ``size`` NDC units across, scattered over and just past the screen."""
    centre = torch.rand(batch, num_tri, 1, 2, generator=gen) * 2.2 - 1.1
    offset = (torch.rand(batch, num_tri, 3, 2, generator=gen) * 2 - 1) * size
    xy = (centre + offset).reshape(batch, 3 * num_tri, 2)
    z = torch.rand(batch, 3 * num_tri, 1, generator=gen) * 1.8 - 0.9
    w = torch.rand(batch, 3 * num_tri, 1, generator=gen) + 1.0
    pos = torch.cat([xy * w, z * w, w], -1)
    tri = torch.arange(3 * num_tri, dtype=torch.int32).view(num_tri, 3)
    return pos, tri


def grid_mesh(n, gen, batch=1, jitter=0.02):
    """A connected ``n x n`` quad grid over most of the screen, randomly tilted in depth."""
    lin = torch.linspace(-0.9, 0.9, n + 1)
    gy, gx = torch.meshgrid(lin, lin, indexing="ij")
    xy = torch.stack([gx, gy], -1).reshape(-1, 2)
    xy = xy[None].expand(batch, -1, -1) + torch.randn(batch, xy.shape[0], 2, generator=gen) * jitter
    z = torch.rand(batch, 1, 1, generator=gen) * 0.6 - 0.3 + xy[..., :1] * 0.3
    w = 1.0 + 0.3 * torch.rand(batch, xy.shape[1], 1, generator=gen)
    pos = torch.cat([xy * w, z * w, w], -1)
    idx = torch.arange((n + 1) * (n + 1)).view(n + 1, n + 1)
    a, b, c, d = (t.flatten() for t in (idx[:-1, :-1], idx[:-1, 1:], idx[1:, 1:], idx[1:, :-1]))
    tri = torch.cat([torch.stack([a, b, c], -1), torch.stack([a, c, d], -1)]).int()
    return pos.contiguous(), tri


# --------------------------------------------------------------------------------------------
# Meshes and cameras of the benchmark configurations
# --------------------------------------------------------------------------------------------

_ICO_VERTS = None


def icosphere(subdivisions: int):
    """Unit icosphere: ``(positions [V, 3] float32, tri [T, 3] int32)``, 20 * 4**s triangles.

    Built by repeated midpoint subdivision with shared edge vertices and re-normalisation
    (642 vertices / 1280 triangles at 3, 655362 / 1310720 at 8).
    """
    g = (1 + math.sqrt(5)) / 2
    verts = torch.tensor(
        [[-1, g, 0], [1, g, 0], [-1, -g, 0], [1, -g, 0], [0, -1, g], [0, 1, g],
         [0, -1, -g], [0, 1, -g], [g, 0, -1], [g, 0, 1], [-g, 0, -1], [-g, 0, 1]],
        dtype=torch.float64,
    )  # fmt: skip
    faces = torch.tensor(
        [[0, 11, 5], [0, 5, 1], [0, 1, 7], [0, 7, 10], [0, 10, 11], [1, 5, 9], [5, 11, 4],
         [11, 10, 2], [10, 7, 6], [7, 1, 8], [3, 9, 4], [3, 4, 2], [3, 2, 6], [3, 6, 8],
         [3, 8, 9], [4, 9, 5], [2, 4, 11], [6, 2, 10], [8, 6, 7], [9, 8, 1]]
    )  # fmt: skip
    verts = F.normalize(verts, dim=-1)
    for _ in range(subdivisions):
        e = torch.cat([faces[:, [0, 1]], faces[:, [1, 2]], faces[:, [2, 0]]]).sort(-1).values
        unique, inverse = torch.unique(e, dim=0, return_inverse=True)
        mid = inverse.view(3, -1) + verts.shape[0]
        verts = F.normalize(torch.cat([verts, verts[unique].mean(1)]), dim=-1)
        a, b, c = faces.unbind(-1)
        ab, bc, ca = mid
        faces = torch.cat(
            [torch.stack([a, ab, ca], -1), torch.stack([b, bc, ab], -1),
             torch.stack([c, ca, bc], -1), torch.stack([ab, bc, ca], -1)]
        )  # fmt: skip
    return verts.float(), faces.int()


def torus_knot(p: int, q: int, segments: int, sides: int, radius=1.0, tube=0.3):
    """Tube of radius ``tube`` around a ``(p, q)`` torus knot of major radius ``radius``.

    Returns ``(positions [segments * sides, 3], tri [2 * segments * sides, 3])``.
    """
    t = torch.arange(segments, dtype=torch.float64) / segments * 2 * math.pi

    def curve(s):
        r = radius * (2 + torch.cos(q * s)) / 3
        return torch.stack([r * torch.cos(p * s), r * torch.sin(p * s), -radius * torch.sin(q * s) / 3], -1)

    h = 1e-4
    c0, c1, cm = curve(t), curve(t + h), curve(t - h)
    tangent = F.normalize(c1 - cm, dim=-1)
    bend = c1 - 2 * c0 + cm
    normal = F.normalize(bend - (bend * tangent).sum(-1, keepdim=True) * tangent, dim=-1)
    binormal = torch.linalg.cross(tangent, normal, dim=-1)
    ang = torch.arange(sides, dtype=torch.float64) / sides * 2 * math.pi
    around = torch.cos(ang)[:, None] * normal[:, None] + torch.sin(ang)[:, None] * binormal[:, None]
    verts = (c0[:, None] + tube * around).reshape(-1, 3).float()
    i, j = torch.meshgrid(torch.arange(segments), torch.arange(sides), indexing="ij")
    i, j = i.flatten(), j.flatten()

    def index(a, b):
        return (a % segments) * sides + b % sides

    a, b, c, d = index(i, j), index(i + 1, j), index(i + 1, j + 1), index(i, j + 1)
    tri = torch.cat([torch.stack([a, c, b], -1), torch.stack([a, d, c], -1)]).int()
    return verts, tri


def perspective(fov_y_deg: float, aspect: float = 1.0, near: float = 0.1, far: float = 10.0):
    """OpenGL projection matrix ``[4, 4]``."""
    f = 1 / math.tan(math.radians(fov_y_deg) / 2)
    return torch.tensor(
        [[f / aspect, 0, 0, 0], [0, f, 0, 0],
         [0, 0, (far + near) / (near - far), 2 * far * near / (near - far)], [0, 0, -1, 0]],
        dtype=torch.float32,
    )  # fmt: skip


def look_at(eye):
    """View matrices ``[B, 4, 4]`` for cameras at ``eye [B, 3]`` looking at the origin."""
    up = eye.new_tensor([0.0, 1.0, 0.0]).expand_as(eye)
    fwd = F.normalize(-eye, dim=-1)
    right = F.normalize(torch.linalg.cross(fwd, up, dim=-1), dim=-1)
    true_up = torch.linalg.cross(right, fwd, dim=-1)
    rot = torch.stack([right, true_up, -fwd], -2)
    view = torch.eye(4).repeat(eye.shape[0], 1, 1)
    view[:, :3, :3] = rot
    view[:, :3, 3] = -(rot @ eye[..., None]).squeeze(-1)
    return view


def orbit_cameras(views: int, distance: float, gen) -> torch.Tensor:
    """Random camera positions on a sphere of radius ``distance``, pitch within +-60 degrees."""
    yaw = torch.rand(views, generator=gen) * 2 * math.pi
    pitch = (torch.rand(views, generator=gen) * 2 - 1) * math.radians(60)
    return distance * torch.stack(
        [torch.sin(yaw) * torch.cos(pitch), torch.sin(pitch), torch.cos(yaw) * torch.cos(pitch)], -1
    )


def to_clip(verts, mvp):
    """``[V, 3]`` world positions to ``[B, V, 4]`` clip space under ``mvp [B, 4, 4]``."""
    homo = F.pad(verts, (0, 1), value=1.0)
    return (homo @ mvp.transpose(-1, -2)).contiguous()


def random_rotation(gen):
    q = F.normalize(torch.randn(4, generator=gen), dim=0)
    w, x, y, z = q.tolist()
    return torch.tensor(
        [[1 - 2 * (y * y + z * z), 2 * (x * y - z * w), 2 * (x * z + y * w)],
         [2 * (x * y + z * w), 1 - 2 * (x * x + z * z), 2 * (y * z - x * w)],
         [2 * (x * z - y * w), 2 * (y * z + x * w), 1 - 2 * (x * x + y * y)]],
    )  # fmt: skip


def spherical_uv(verts):
    """``[V, 2]`` longitude/latitude texture coordinates of unit-sphere positions."""
    x, y, z = verts.unbind(-1)
    u = torch.atan2(x, z) / (2 * math.pi) + 0.5
    v = torch.acos(y.clamp(-1, 1)) / math.pi
    return torch.stack([u, v], -1).float()


def displaced_grid(num_tri: int, views: int):
    """The scene of the reference's rasterize and pipeline benchmarks
    (benchmarks/bench_rasterize.py:19-53, bench_pipeline.py:25-28), restated.

    An ``(n + 1)^2``-vertex grid over ``[-1, 1]^2`` in the x-z plane, ``n = round(sqrt(num_tri /
    2))``, lifted by ``y = 0.1 sin(6x) cos(5z)``, two triangles per cell (all cells' ``(a, b, d)``
    triangles, then all their ``(a, d, c)`` ones), seen by ``views`` cameras turned about the y
    axis in equal steps, moved by ``(0, -0.6, 2.2)`` and projected with focal length 1.5, near
    0.1 and far 10 (``w`` is the camera-space z). Returns clip positions ``[views, V, 4]``, ``tri``
    and the planar texture coordinates ``((x + 1) / 2, (z + 1) / 2)`` of each vertex.
    """
    n = max(1, round(math.sqrt(num_tri / 2)))
    s = torch.linspace(-1, 1, n + 1)
    z, x = torch.meshgrid(s, s, indexing="ij")  # vertex i * (n + 1) + j sits at (s[j], s[i])
    world = torch.stack([x, 0.1 * torch.sin(6 * x) * torch.cos(5 * z), z], -1).reshape(-1, 3)
    idx = torch.arange((n + 1) ** 2).view(n + 1, n + 1)
    a, b = idx[:-1, :-1], idx[:-1, 1:]
    c, d = idx[1:, :-1], idx[1:, 1:]
    tri = torch.cat([torch.stack([a, b, d], -1), torch.stack([a, d, c], -1)]).reshape(-1, 3).int()
    near, far, focal = 0.1, 10.0, 1.5
    project = torch.tensor([[focal, 0, 0, 0], [0, focal, 0, 0],
                            [0, 0, (far + near) / (far - near), -2 * far * near / (far - near)],
                            [0, 0, 1, 0]])  # fmt: skip
    clips = []
    for k in range(views):
        angle = 2 * math.pi * k / max(views, 1)
        turn = torch.eye(4)
        turn[0, 0], turn[0, 2] = math.cos(angle), math.sin(angle)
        turn[2, 0], turn[2, 2] = -math.sin(angle), math.cos(angle)
        turn[:3, 3] = torch.tensor([0.0, -0.6, 2.2])
        clips.append(to_clip(world, (project @ turn)[None])[0])
    t = torch.linspace(0, 1, n + 1)
    tv, tu = torch.meshgrid(t, t, indexing="ij")
    uv = torch.stack([tu, tv], -1).reshape(-1, 2)
    return torch.stack(clips).contiguous(), tri, uv.contiguous()


def config1_scene(seed=0):
    """icosphere-3 under a random rotation, 1 view at 256x256."""
    gen = torch.Generator().manual_seed(seed)
    verts, tri = icosphere(3)
    rot = random_rotation(gen)
    world = verts @ rot.T
    eye = torch.tensor([[0.0, 0.0, 3.0]])
    mvp = perspective(45.0, 1.0, 0.1, 10.0) @ look_at(eye)
    pos = to_clip(world, mvp)
    uv = spherical_uv(verts)
    tex = torch.rand(1, 256, 256, 3, generator=gen)
    target = torch.rand(1, 256, 256, 3, generator=gen)
    return dict(pos=pos, tri=tri, uv=uv, tex=tex, target=target, resolution=(256, 256))


def config5_scene(views=64, resolution=1024, subdivisions=8, tex_size=4096, seed=5):
    """displaced icosphere-8, random orbit cameras, 4096^2 x 3 texture.

    Returns CPU tensors; ``attr`` holds ``[u, v, nx, ny, nz]`` per vertex.
    """
    gen = torch.Generator().manual_seed(seed)
    verts, tri = icosphere(subdivisions)
    normals = verts.clone()
    world = verts * (1 + 0.01 * torch.randn(verts.shape[0], 1, generator=gen))
    eye = orbit_cameras(views, 3.0, gen)
    mvp = perspective(45.0, 1.0, 0.1, 10.0) @ look_at(eye)
    pos = to_clip(world, mvp)
    attr = torch.cat([spherical_uv(verts), normals], -1).contiguous()
    tex = torch.rand(1, tex_size, tex_size, 3, generator=gen)
    return dict(pos=pos, tri=tri, attr=attr, tex=tex, resolution=(resolution, resolution), gen=gen,
                world=world, mvp=mvp)


# Reduced versions of BASELINE configs 2-5 for parity tests against the CPU oracle: the same
# generators and parameters, fewer views, triangles and pixels, so that the oracle's brute-force
# visibility finishes in seconds.


def config2_small(views=2, resolution=64, segments=96, sides=12, seed=2):
    """Config 2 shape: (2, 3) torus knot with N(0, 0.01) jitter, orbit cameras at distance 4,
    fov 40 degrees; rasterize only, with N(0, 1) upstream gradients on rast and rast_db."""
    gen = torch.Generator().manual_seed(seed)
    verts, tri = torus_knot(2, 3, segments, sides)
    verts = verts + 0.01 * torch.randn(verts.shape, generator=gen)
    mvp = perspective(40.0) @ look_at(orbit_cameras(views, 4.0, gen))
    pos = to_clip(verts, mvp)
    g_rast = torch.randn(views, resolution, resolution, 4, generator=gen)
    g_db = torch.randn(views, resolution, resolution, 4, generator=gen)
    return dict(pos=pos, tri=tri, resolution=(resolution, resolution), g_rast=g_rast, g_db=g_db)


def config3_small(views=2, resolution=64, subdivisions=3, tex_size=64, seed=3):
    """Config 3 shape: icosphere with N(0, 0.02) radial displacement, random orbit cameras,
    attr = [u, v, 8 channels N(0, 1)] with all channels differentiated, a 4-channel texture
    sampled trilinearly through a texture_construct_mip stack."""
    gen = torch.Generator().manual_seed(seed)
    verts, tri = icosphere(subdivisions)
    world = verts * (1 + 0.02 * torch.randn(verts.shape[0], 1, generator=gen))
    mvp = perspective(45.0) @ look_at(orbit_cameras(views, 3.0, gen))
    pos = to_clip(world, mvp)
    attr = torch.cat([spherical_uv(verts), torch.randn(verts.shape[0], 8, generator=gen)], -1)
    tex = torch.rand(1, tex_size, tex_size, 4, generator=gen)
    target = torch.rand(views, resolution, resolution, 4, generator=gen)
    return dict(pos=pos, tri=tri, attr=attr.contiguous(), tex=tex, target=target,
                resolution=(resolution, resolution))


def config4_small(views=2, resolution=48, segments=64, sides=10, cube_size=16, layers=4, seed=4):
    """Config 4 shape: (3, 4) torus knot, a [1, 6, s, s, 3] cube map looked up with interpolated
    normals (directions) and their screen derivatives, antialiasing, and depth peeling."""
    gen = torch.Generator().manual_seed(seed)
    verts, tri = torus_knot(3, 4, segments, sides)
    mvp = perspective(45.0) @ look_at(orbit_cameras(views, 3.5, gen))
    pos = to_clip(verts, mvp)
    normals = F.normalize(verts - verts.mean(0, keepdim=True), dim=-1)
    cube = torch.rand(1, 6, cube_size, cube_size, 3, generator=gen)
    target = torch.rand(views, resolution, resolution, 3, generator=gen)
    return dict(pos=pos, tri=tri, normals=normals.contiguous(), cube=cube, target=target,
                resolution=(resolution, resolution), layers=layers)


def config5_small(views=2, resolution=64, subdivisions=4, noise=0.15, tex_size=64, seed=5):
    """Config 5 character at small size: an icosphere whose radial N(0, noise) displacement is
    about twice its edge length (as N(0, 0.01) is for icosphere-8), so that triangles are spiky
    and overlap several deep, with attr [u, v, normal], a trilinear texture and antialiasing."""
    gen = torch.Generator().manual_seed(seed)
    verts, tri = icosphere(subdivisions)
    world = verts * (1 + noise * torch.randn(verts.shape[0], 1, generator=gen))
    mvp = perspective(45.0) @ look_at(orbit_cameras(views, 3.0, gen))
    pos = to_clip(world, mvp)
    attr = torch.cat([spherical_uv(verts), verts], -1).contiguous()
    tex = torch.rand(1, tex_size, tex_size, 3, generator=gen)
    target = torch.rand(views, resolution, resolution, 3, generator=gen)
    return dict(pos=pos, tri=tri, attr=attr, tex=tex, target=target,
                resolution=(resolution, resolution))
