"""The bounds-checked build (DIFFRAST_B200_CHECK=1) on the GPU, in a child process.

1. The config-5-character pipeline (rasterize, interpolate, trilinear texture, antialias with the
   fused loss, backward) and a cube-map lookup run with every data-dependent index checked and no
   fault recorded, giving the ordinary build's results (ids and images identical, gradients
   within 1e-5 relative: atomics add in another order).
2. A vertex index past the end of pos, planted in tri behind the host's index check (which would
   refuse it with a ValueError), reaches the visibility and resolve kernels of the checked build:
   each check that sees it records it and sends the access to element 0, so nothing reads out of
   bounds, and the call raises BoundsFault naming the site and the index. The same process then
   rasterizes correct input without a fault.
"""

import subprocess
import sys
import textwrap
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
pytestmark = pytest.mark.gpu

PIPELINE = textwrap.dedent(
    """
    import sys, torch
    sys.path.insert(0, {root!r}); sys.path.insert(0, {tests!r})
    import diffrast_b200 as dr, scenes
    from diffrast_b200 import _native
    assert _native.lib().dr_checked_build() == {checked}
    sc = scenes.config5_small(views=2)
    ctx = dr.RasterizeContext("cuda")
    pos = sc["pos"].cuda().requires_grad_(True)
    tex = sc["tex"].cuda().requires_grad_(True)
    tri, attr, target = sc["tri"].cuda(), sc["attr"].cuda(), sc["target"].cuda()
    rast, rast_db = dr.rasterize(ctx, pos, tri, sc["resolution"])
    out, out_da = dr.interpolate(attr, rast, tri, rast_db=rast_db, diff_attrs="all")
    color = dr.texture(tex, out[..., 0:2], out_da[..., 0:4], filter_mode="linear-mipmap-linear")
    image, loss = dr.antialias_mse(color, rast, pos, tri, target)
    loss.backward()
    cube = torch.rand(1, 6, 16, 16, 3, generator=torch.Generator().manual_seed(3)).cuda()
    dirs = torch.nn.functional.normalize(out[..., 2:5].detach(), dim=-1).contiguous()
    env = dr.texture(cube, dirs, filter_mode="linear", boundary_mode="cube")
    _native.check_faults()
    torch.save(dict(ids=rast[..., 3].cpu(), image=image.detach().cpu(), env=env.cpu(),
                    g_pos=pos.grad.cpu(), g_tex=tex.grad.cpu()), {out!r})
    """
)

PLANTED = textwrap.dedent(
    """
    import sys, torch
    sys.path.insert(0, {root!r}); sys.path.insert(0, {tests!r})
    import diffrast_b200 as dr, scenes
    from diffrast_b200 import _native, ops
    sc = scenes.config5_small(views=1)
    ctx = dr.RasterizeContext("cuda")
    pos, tri = sc["pos"].cuda(), sc["tri"].clone()
    bad = pos.shape[1] + 1000
    tri[5, 1] = bad
    ops._check_indices = lambda tri, num_vert: None  # let the bad index reach the kernels
    try:
        dr.rasterize(ctx, pos, tri.cuda(), sc["resolution"])
    except _native.BoundsFault as fault:
        print("FAULT", fault.site, fault.index)
    else:
        print("NO FAULT")
    rast, _ = dr.rasterize(ctx, pos, sc["tri"].cuda(), sc["resolution"])
    _native.check_faults()
    print("CLEAN", int((rast[..., 3] > 0).sum()))
    """
)


def run_child(script: str, checked: bool, tmp_path, name: str):
    out = tmp_path / f"{name}.pt"
    code = script.format(root=str(ROOT), tests=str(ROOT / "tests"), checked=int(checked),
                         out=str(out))
    env = {"DIFFRAST_B200_CHECK": "1" if checked else "0", "PATH": "/usr/bin:/bin"}
    done = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True,
                          timeout=600, env=env)
    assert done.returncode == 0, done.stderr[-3000:]
    return done.stdout, out


def test_checked_pipeline_records_no_fault_and_matches_ordinary_build(tmp_path):
    _, checked = run_child(PIPELINE, True, tmp_path, "checked")
    _, ordinary = run_child(PIPELINE, False, tmp_path, "ordinary")
    a, b = torch.load(checked), torch.load(ordinary)
    assert torch.equal(a["ids"], b["ids"]) and (a["ids"] > 0).any()
    assert torch.equal(a["image"], b["image"]) and torch.equal(a["env"], b["env"])
    for key in ("g_pos", "g_tex"):
        scale = max(1.0, b[key].abs().max().item())
        torch.testing.assert_close(a[key], b[key], atol=1e-5 * scale, rtol=1e-5)


def test_planted_vertex_index_is_reported_not_read(tmp_path):
    stdout, _ = run_child(PLANTED, True, tmp_path, "planted")
    lines = stdout.strip().splitlines()
    fault = next(line for line in lines if line.startswith(("FAULT", "NO FAULT")))
    assert fault.startswith("FAULT vertex index read from tri"), stdout
    num_vert = int(fault.split()[-1]) - 1000
    assert num_vert > 0
    clean = next(line for line in lines if line.startswith("CLEAN"))
    assert int(clean.split()[1]) > 0
