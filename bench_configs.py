#!/usr/bin/env python
"""Both arms on one B200, case by case: this library and the reference's Triton backend
(unmodified, from ``baseline/_ref``), on BASELINE configurations 1-4 at their stated sizes and on
the reference's own pipeline benchmark grid (benchmarks/bench_pipeline.py:21-44 of the reference:
a displaced grid of 10k, 100k and 1M triangles seen by 8 views at 256^2 to 2048^2, planar texture
coordinates, a 1024^2 x 3 texture sampled linear-mipmap-linear, antialias, ``sum().backward()``
to positions and texture). Configuration 5, the scaling workload, is bench.py's.

Each case builds its inputs once on the device and runs the same op sequence through both
packages. Times follow the reference's benchmarks (bench_rasterize.py:56-72 there): warm-up, then
the median of individually synchronised steps, each step bracketed by CUDA events. This library's
arm is timed eagerly (as the reference's API runs) and again replaying a CUDA graph of the step.
One JSON line per case:

    python bench_configs.py [--cases c1 c2 c3 c4 grid] [--repeats 10] [--warmup-s 2] [--no-triton]
"""

from __future__ import annotations

import argparse
import json
import statistics
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))

import torch  # noqa: E402
import torch.nn.functional as F  # noqa: E402

import scenes  # noqa: E402
from bench import UNIT, ClockSampler, gpu_id, reference_package  # noqa: E402

GRID_TRIANGLES = (10_000, 100_000, 1_000_000)
GRID_RESOLUTIONS = (256, 512, 1024, 2048)


def median_ms(fn, repeats: int, warmup_s: float) -> float:
    fn()
    torch.cuda.synchronize()
    start = time.perf_counter()
    while time.perf_counter() - start < warmup_s:
        fn()
        torch.cuda.synchronize()
    times = []
    for _ in range(repeats):
        begin, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        begin.record()
        fn()
        end.record()
        end.synchronize()
        times.append(begin.elapsed_time(end))
    return statistics.median(times)


def graph_ms(fn, ctx, repeats: int) -> tuple[float | None, str | None]:
    """Median of individually synchronised replays of a CUDA graph of ``fn`` (this library only),
    or None and the reason when the step does not capture."""
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    try:
        with torch.cuda.stream(stream):
            for _ in range(2):
                fn()
            with torch.cuda.graph(graph, stream=stream):
                fn()
    except Exception as exc:  # noqa: BLE001 - any capture failure: report it, time eagerly only
        torch.cuda.synchronize()
        return None, str(exc).splitlines()[0][:200]
    torch.cuda.current_stream().wait_stream(stream)
    ms = median_ms(graph.replay, repeats, 0.5)
    overflowed = ctx.capture_overflowed()
    graph.reset()
    if overflowed:
        return None, "a captured visibility pass outgrew its binning capacity"
    return ms, None


# Each case: (name, pixels per step, description, make) where make(api, ctx) returns the step
# functions {"fwd_bwd": f} (and "fwd" for the grid) over inputs built on the device.


def case_c1(dev):
    sc = scenes.config1_scene(seed=0)
    res = sc["resolution"]

    def make(api, ctx):
        pos = sc["pos"].to(dev).requires_grad_(True)
        tex = sc["tex"].to(dev).requires_grad_(True)
        tri, uv, target = sc["tri"].to(dev), sc["uv"].to(dev), sc["target"].to(dev)

        def fwd_bwd():
            pos.grad = tex.grad = None
            rast, _ = api.rasterize(ctx, pos, tri, res)
            uvp, _ = api.interpolate(uv, rast, tri)
            color = api.texture(tex, uvp, filter_mode="linear")
            image = api.antialias(color, rast, pos, tri)
            F.mse_loss(image, target).backward()

        return {"fwd_bwd": fwd_bwd}

    return ("c1", res[0] * res[1], "BASELINE config 1: 1 view 256x256, icosphere-3, tex 256^2x3 "
            "linear, antialias, MSE, backward to tex and pos", make)


def case_c2(dev, views=8, size=1024, segments=512, sides=64):
    sc = scenes.config2_small(views=views, resolution=size, segments=segments, sides=sides)
    res = sc["resolution"]

    def make(api, ctx):
        pos = sc["pos"].to(dev).requires_grad_(True)
        tri = sc["tri"].to(dev)
        g_rast, g_db = sc["g_rast"].to(dev), sc["g_db"].to(dev)

        def fwd_bwd():
            pos.grad = None
            rast, rast_db = api.rasterize(ctx, pos, tri, res)
            torch.autograd.backward([rast, rast_db], [g_rast, g_db])

        return {"fwd_bwd": fwd_bwd}

    return ("c2", views * res[0] * res[1], "BASELINE config 2: 8 views 1024x1024, (2,3) torus knot "
            "512x64 (65536 tris) with N(0,0.01) jitter, rasterize only, N(0,1) upstream gradients "
            "on rast and rast_db, backward to pos", make)


def case_c3(dev, views=16, size=512, subdivisions=6, tex_size=2048):
    sc = scenes.config3_small(views=views, resolution=size, subdivisions=subdivisions,
                              tex_size=tex_size)
    res = sc["resolution"]

    def make(api, ctx):
        pos = sc["pos"].to(dev)
        tri = sc["tri"].to(dev)
        attr = sc["attr"].to(dev).requires_grad_(True)
        tex = sc["tex"].to(dev).requires_grad_(True)
        target = sc["target"].to(dev)

        def fwd_bwd():
            attr.grad = tex.grad = None
            rast, rast_db = api.rasterize(ctx, pos, tri, res)
            out, out_da = api.interpolate(attr, rast, tri, rast_db=rast_db, diff_attrs="all")
            stack = api.texture_construct_mip(tex)
            color = api.texture(tex, out[..., 0:2], out_da[..., 0:4], mip=stack,
                                filter_mode="linear-mipmap-linear")
            loss = F.mse_loss(color, target) + out[..., 2:].square().mean()
            loss.backward()

        return {"fwd_bwd": fwd_bwd}

    return ("c3", views * res[0] * res[1], "BASELINE config 3: 16 views 512x512, icosphere-6 "
            "(81920 tris) with N(0,0.02) displacement, attr [u, v, 8 x N(0,1)] diff_attrs all, "
            "tex 2048^2x4 linear-mipmap-linear through texture_construct_mip, MSE on the colour "
            "plus the mean square of the 8 attribute channels, backward to tex and attr (via uv, "
            "uv_da and the channels)", make)


def reflect(n, n_da, p, p_da, eye):
    """Directions ``r = v - 2 (v . n) n`` for view vectors ``v = p - eye`` and their screen
    derivatives from those of ``n`` and ``p`` (``*_da``: ``[..., 6]`` as (d/dX, d/dY) per
    component)."""
    v = p - eye[:, None, None, :]
    n_d = n_da.unflatten(-1, (3, 2))
    p_d = p_da.unflatten(-1, (3, 2))
    vn = (v * n).sum(-1, keepdim=True)
    r = v - 2 * vn * n
    vn_d = (p_d * n[..., None]).sum(-2) + (v[..., None] * n_d).sum(-2)
    r_d = p_d - 2 * (vn_d[..., None, :] * n[..., None] + vn[..., None] * n_d)
    return r, r_d.flatten(-2)


def case_c4(dev, views=8, size=512, segments=400, sides=64, cube_size=512):
    res, layers = (size, size), 4
    gen = torch.Generator().manual_seed(4)
    verts, tri_cpu = scenes.torus_knot(3, 4, segments, sides)
    eye_cpu = scenes.orbit_cameras(views, 3.5, gen)
    mvp = scenes.perspective(45.0) @ scenes.look_at(eye_cpu)
    pos_cpu = scenes.to_clip(verts, mvp)
    normals = F.normalize(verts - verts.mean(0, keepdim=True), dim=-1)
    attr_cpu = torch.cat([normals, verts], -1).contiguous()
    cube_cpu = torch.rand(1, 6, cube_size, cube_size, 3, generator=gen)
    target_cpu = torch.rand(views, *res, 3, generator=gen)

    def make(api, ctx):
        pos = pos_cpu.to(dev).requires_grad_(True)
        cube = cube_cpu.to(dev).requires_grad_(True)
        tri, attr = tri_cpu.to(dev), attr_cpu.to(dev)
        eye, target = eye_cpu.to(dev), target_cpu.to(dev)

        def fwd_bwd():
            pos.grad = cube.grad = None
            loss = 0.0
            with api.DepthPeeler(ctx, pos, tri, res) as peeler:
                for _ in range(layers):
                    rast, rast_db = peeler.rasterize_next_layer()
                    out, out_da = api.interpolate(attr, rast, tri, rast_db=rast_db, diff_attrs="all")
                    dirs, dirs_da = reflect(out[..., 0:3], out_da[..., 0:6], out[..., 3:6],
                                            out_da[..., 6:12], eye)
                    color = api.texture(cube, dirs, dirs_da, filter_mode="linear-mipmap-linear",
                                        boundary_mode="cube")
                    image = api.antialias(color, rast, pos, tri)
                    loss = loss + F.mse_loss(image, target)
            loss.backward()

        return {"fwd_bwd": fwd_bwd}

    return ("c4", views * res[0] * res[1], "BASELINE config 4: 8 views 512x512, (3,4) torus knot "
            "400x64 (51200 tris), 4 depth-peeled layers, each: interpolate [normal, position] "
            "diff_attrs all, view vectors reflected about the interpolated normals (with their "
            "screen derivatives, torch ops), cube [1,6,512,512,3] linear-mipmap-linear, antialias, "
            "MSE; backward to cube and pos; pixels counted once per view", make)


def case_grid(dev, num_tri, res):
    views = 8
    pos_cpu, tri_cpu, uv_cpu = scenes.displaced_grid(num_tri, views)
    tex_cpu = torch.rand(1, 1024, 1024, 3, generator=torch.Generator().manual_seed(0))

    def make(api, ctx):
        pos = pos_cpu.to(dev).requires_grad_(True)
        tex = tex_cpu.to(dev).requires_grad_(True)
        tri, uv = tri_cpu.to(dev), uv_cpu.to(dev)

        def render():
            rast, rast_db = api.rasterize(ctx, pos, tri, (res, res))
            out, out_da = api.interpolate(uv, rast, tri, rast_db=rast_db, diff_attrs="all")
            color = api.texture(tex, out, out_da, filter_mode="linear-mipmap-linear")
            return api.antialias(color, rast, pos, tri)

        def fwd():
            with torch.no_grad():
                render()

        def fwd_bwd():
            pos.grad = tex.grad = None
            render().sum().backward()

        return {"fwd": fwd, "fwd_bwd": fwd_bwd}

    return (f"grid_{num_tri // 1000}k_{res}", views * res * res,
            f"the reference's pipeline benchmark: displaced grid {tri_cpu.shape[0]} tris, {views} "
            f"views {res}x{res}, planar uv diff_attrs all, tex 1024^2x3 linear-mipmap-linear, "
            "antialias, sum().backward() to pos and tex", make)


def run_case(case, dev, ours, ref, repeats: int, warmup_s: float) -> dict:
    name, pixels, what, make = case
    line = {"case": name, "workload": what, "pixels_per_step": pixels, "unit": UNIT}
    arms = [("ours", ours)] + ([("triton", ref)] if ref is not None else [])
    for arm, api in arms:
        ctx = api.RasterizeContext(dev)
        fns = make(api, ctx)
        result = {}
        try:
            for kind, fn in fns.items():
                ms = median_ms(fn, repeats, warmup_s)
                result[kind] = {"ms": round(ms, 3), "value": round(pixels / (ms / 1e3) / 1e6, 1)}
            if arm == "ours":
                ms, why = graph_ms(fns["fwd_bwd"], ctx, repeats)
                result["fwd_bwd_graph"] = (
                    {"ms": round(ms, 3), "value": round(pixels / (ms / 1e3) / 1e6, 1)}
                    if ms is not None else {"unavailable": why})  # fmt: skip
        except torch.OutOfMemoryError:
            result["unavailable"] = "out of device memory"
        result["peak_mem_gb"] = round(torch.cuda.max_memory_allocated(dev) / 1e9, 2)
        line[arm] = result
        del fns, ctx
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        torch.cuda.reset_peak_memory_stats(dev)
    if ref is None:
        line["triton"] = {"unavailable": "not run (--no-triton) or the reference package is not "
                                         "installed under baseline/_ref"}
    ours_v = line["ours"].get("fwd_bwd", {}).get("value")
    ref_v = line["triton"].get("fwd_bwd", {}).get("value")
    if ours_v and ref_v:
        line["speedup_fwd_bwd_eager"] = round(ours_v / ref_v, 2)
    return line


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--cases", nargs="+", default=["c1", "c2", "c3", "c4", "grid"])
    parser.add_argument("--repeats", type=int, default=10)
    parser.add_argument("--warmup-s", type=float, default=2.0)
    parser.add_argument("--no-triton", action="store_true", help="time this library's arm only")
    args = parser.parse_args()
    if not torch.cuda.is_available():
        raise SystemExit("bench_configs.py needs a CUDA device")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    import diffrast_b200 as ours

    ref = None if args.no_triton else reference_package("triton")
    cases = []
    for name in args.cases:
        if name == "grid":
            cases += [case_grid(dev, t, r) for t in GRID_TRIANGLES for r in GRID_RESOLUTIONS]
        else:
            cases.append({"c1": case_c1, "c2": case_c2, "c3": case_c3, "c4": case_c4}[name](dev))
    for case in cases:
        with ClockSampler(gpu_id(dev)) as clocks:
            line = run_case(case, dev, ours, ref, args.repeats, args.warmup_s)
        line["clocks"] = clocks.summary()
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
