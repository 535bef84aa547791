#!/usr/bin/env python
"""Benchmark of the differentiable render path: rasterize -> interpolate -> texture -> antialias,
forward and backward, in Mpixel/s, on BASELINE configuration 5.

Workload (synthetic, seeded): icosphere level 8 (655,362 vertices, 1,310,720 triangles) with
N(0, 0.01) radial displacement, 64 random orbit cameras at 1024x1024, interpolation of
[u, v, nx, ny, nz] with all derivatives, a 4096x4096x3 uniform texture sampled trilinearly
(its mip chain rebuilt every step, as the texture requires gradients), antialiasing, MSE against
a random target, backward to the texture and the world-space vertex positions. The mesh and the
texture are parameters resident on the GPU; each step's inputs are the cameras' matrices and the
target images, and the step starts with the world-to-clip transform (``to_clip``). The 64 views
are sharded across the ranks (strong scaling); the texture and position gradients are summed with
NCCL all-reduces.

    python bench.py [--gpus N --steps K --warmup W] [--impl reference | --impl triton]

One JSON line is printed by rank 0. ``--impl reference`` times the reference's CPU backend (the
unmodified reference package when it is installed under ``baseline/_ref``, else the golden-pinned
CPU restatement in ``oracle/``) with all host threads on a bounded sample of the same workload.
``--impl triton`` times the reference's own GPU backend (Triton, unmodified, from
``baseline/_ref``) on the same workload on one GPU; the default run does that too, in a
subprocess, and reports it as ``gpu_reference``, together with a same-configuration pair on
BASELINE configuration 1 (this library on the GPU against the reference's CPU backend).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

METRIC = "fwd+bwd Mpixel/s of rasterize→interpolate→texture→antialias at 1/2/4/8 B200"
UNIT = "Mpixel/s"
ATTR_CHANNELS, DIFF_CHANNELS, TEX_CHANNELS = 5, 5, 3
# Kernels each wrapper launches per call (the visibility stage adds 4 when it bins triangles; the
# mip stages depend on the texture size, see mip_launches).
LAUNCHES = {
    "raster_visibility": 2, "resolve_fwd": 1, "resolve_bwd": 1, "interpolate_fwd": 1,
    "interpolate_bwd": 1, "texture_fwd": 1, "texture_bwd": 1, "mip_build": 1, "mip_adjoint": 1,
    "edge_neighbours": 2, "antialias_fwd": 1, "antialias_bwd": 1, "to_clip_fwd": 1,
    "to_clip_bwd": 1,
}  # fmt: skip


def mip_launches(h: int, w: int, channels: int) -> tuple[int, int]:
    """Kernels of one dr_mip_build call (runs of even halvings, up to six levels per launch, with
    at most 4 channels; one launch per other level) and of one dr_mip_build_bwd call (the same
    steps undone: one launch per run, its 16-byte aligned, at most 4-channel padded gradient
    levels taking the run kernel; one per other level) for an h x w texture's full chain."""
    build, lh, lw = 0, h, w
    while lh > 1 or lw > 1:
        n = 0
        while n < 6 and (lh >> n) % 2 == 0 and (lw >> n) % 2 == 0 and (lh >> n, lw >> n) != (1, 1):
            n += 1
        step = n if n >= 2 and channels <= 4 else 1
        for _ in range(step):
            lh, lw = (lh + 1) // 2, (lw + 1) // 2
        build += 1
    return build, build


def stage_bytes(pixels: int, num_vert: int, views: int, stack_bytes: int, tex_bytes: int,
                fused: int = 0) -> dict:
    """Algorithmic bytes per launch of each stage: API-level tensor reads and writes, fp32.

    Per pixel (C attribute channels, D differentiated channels, Ct texture channels):
    rasterize writes rast + rast_db (32) and its backward reads their gradients (32);
    interpolate reads rast, rast_db (32) and writes 4C + 8D, backward reads 4C + 8D + 32 and writes
    32; texture reads uv, uv_da (24) and writes 4Ct, backward reads 4Ct + 24 and writes 24;
    antialias reads colour and rast (4Ct + 16) and writes 4Ct, backward reads 8Ct + 16 and writes
    4Ct. Per call: clip positions (16 B per vertex and view) for the rasterizer and the transform
    that writes them (its backward reads their gradient), the mip stack for the build and its
    adjoint. With ``fused`` = 1 the texture backward runs the interpolation's backward for the
    coordinates (no interpolation backward launch): it reads the upstream gradient, uv, uv_da and
    rast and writes the gradients of rast and rast_db, 4Ct + 24 + 16 + 32; with 2 the
    rasterizer's backward too (no resolve backward launch): it reads the keys instead of rast and
    writes no per-pixel gradient, 4Ct + 24 + 8, plus the clip positions and their gradient.
    """
    c, d, ct = ATTR_CHANNELS, DIFF_CHANNELS, TEX_CHANNELS
    pos_bytes = views * num_vert * 16
    return {
        "raster_visibility": pos_bytes + pixels * 8,
        "resolve_fwd": pixels * (8 + 32) + pos_bytes,
        "interpolate_fwd": pixels * (32 + 4 * c + 8 * d),
        "mip_build": stack_bytes + tex_bytes,
        "texture_fwd": pixels * (24 + 4 * ct),
        "antialias_fwd": pixels * (16 + 8 * ct),
        "antialias_bwd": pixels * (16 + 12 * ct),
        "texture_bwd": pixels * (48 + 4 * ct, 4 * ct + 24 + 16 + 32, 4 * ct + 24 + 8)[fused]
                       + 2 * tex_bytes + (2 * pos_bytes if fused == 2 else 0),
        "mip_adjoint": 2 * stack_bytes + tex_bytes,
        "interpolate_bwd": pixels * (64 + 4 * c + 8 * d),
        "resolve_bwd": pixels * (8 + 32) + 2 * pos_bytes,
        "to_clip_fwd": pos_bytes + num_vert * 12,
        "to_clip_bwd": pos_bytes + num_vert * 24,
    }


def step_bytes(pixels, num_vert, views, stack_bytes, tex_bytes) -> int:
    """Whole-step algorithmic bytes: 468 B per pixel at C=5, D=5, Ct=3 plus per-call terms."""
    c, d, ct = ATTR_CHANNELS, DIFF_CHANNELS, TEX_CHANNELS
    per_px = 32 + (32 + 4 * c + 8 * d) + (24 + 4 * ct) + (16 + 8 * ct)
    per_px += (16 + 12 * ct) + (48 + 4 * ct) + (64 + 4 * c + 8 * d) + 32
    return pixels * per_px + views * num_vert * 16 * 7 + num_vert * 36 + 3 * stack_bytes


class ClockSampler:
    """Samples the GPU's SM clock and clock-event (throttle) reasons while active: through NVML
    every 20 ms when the nvidia-ml-py binding loads (read-only queries), else with nvidia-smi every
    200 ms. Nothing is ever set."""

    # NVML clock-event reason bits (nvml.h): the ones a timing must report.
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_uuid: str) -> None:
        self.gpu = gpu_uuid
        self.proc = None
        self.samples: list[tuple[float, float | None, set]] = []
        self.thread = None
        self.stop = threading.Event()
        self.nvml = None

    def __enter__(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            handle = pynvml.nvmlDeviceGetHandleByUUID(self.gpu.encode())
            reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
            self.nvml = (pynvml, handle, reasons)
            self.thread = threading.Thread(target=self._poll_nvml, daemon=True)
        except Exception:  # noqa: BLE001 - no binding or no NVML: fall back to nvidia-smi
            self.nvml = None
            try:
                self.proc = subprocess.Popen(
                    ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                     "--format=csv,noheader,nounits", "-lms", "200"],
                    stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True,
                )  # fmt: skip
                self.thread = threading.Thread(target=self._read_smi, daemon=True)
            except OSError:
                self.proc = None
        if self.thread is not None:
            self.thread.start()
        return self

    def _poll_nvml(self):
        pynvml, handle, reasons = self.nvml
        max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(handle, pynvml.NVML_CLOCK_SM))
        while not self.stop.is_set():
            try:
                mhz = float(pynvml.nvmlDeviceGetClockInfo(handle, pynvml.NVML_CLOCK_SM))
                bits = int(reasons(handle))
            except Exception:  # noqa: BLE001
                break
            self.samples.append((mhz, max_mhz, {n for b, n in self.REASONS.items() if bits & b}))
            self.stop.wait(0.02)

    def _read_smi(self):
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.strip().split(",")]
            if len(parts) < 9:
                continue
            try:
                mhz, max_mhz = float(parts[1]), float(parts[2])
            except ValueError:
                continue
            active = {n for n, flag in zip(names, parts[5:9]) if flag.lower() == "active"}
            self.samples.append((mhz, max_mhz, active))

    def __exit__(self, *exc):
        self.stop.set()
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=2)
        if self.nvml is not None:
            try:
                self.nvml[0].nvmlShutdown()
            except Exception:  # noqa: BLE001
                pass

    def summary(self) -> dict:
        mhz = [m for m, _, _ in self.samples]
        max_mhz = next((x for _, x, _ in self.samples if x), None)
        reasons = set().union(*(r for _, _, r in self.samples)) if self.samples else set()
        return {"sm_mhz": statistics.median(mhz) if mhz else None, "sm_max_mhz": max_mhz,
                "reasons": sorted(reasons), "samples": len(mhz),
                "source": "nvml" if self.nvml is not None else "nvidia-smi"}  # fmt: skip


def measured_traffic(stage: str, pixels: int) -> int | None:
    """DRAM bytes of one launch of `stage`: bytes per pixel from a committed ncu capture
    (profiles/dram_bytes_per_pixel.txt) times the pixels of the launch, or None."""
    per_px = profiled_per_pixel("dram_bytes_per_pixel.txt", stage)
    return None if per_px is None else int(per_px * pixels)


def profiled_per_pixel(name: str, stage: str) -> float | None:
    """Per-pixel figure of `stage` in the committed ncu summary ``profiles/<name>``, or None."""
    path = ROOT / "profiles" / name
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        parts = line.split()
        if len(parts) == 2 and not line.startswith("#") and parts[0] == stage:
            return float(parts[1])
    return None


def issue_roofline(stage: str, pixels: int, ms_per_launch: float, clocks: dict, dev) -> dict | None:
    """Warp-instruction issue rate of one launch of `stage` against the SMs' issue peak (four
    schedulers per SM, one warp instruction each per cycle, at the median SM clock sampled during
    the timing): the bound of a stage that is limited by instructions, not bytes."""
    per_px = profiled_per_pixel("warp_instructions_per_pixel.txt", stage)
    mhz = clocks.get("sm_mhz") or clocks.get("sm_max_mhz")
    if per_px is None or not mhz:
        return None
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    achieved = per_px * pixels / (ms_per_launch / 1e3)
    peak = sms * 4 * mhz * 1e6
    return {"bound": "issue", "kernel": stage, "achieved": round(achieved / 1e9, 1),
            "peak": round(peak / 1e9, 1), "unit": "G warp instructions/s",
            "frac": round(achieved / peak, 4),
            "instructions_source": "ncu smsp__inst_executed.sum per pixel on the 8-view case "
                                   "(profiles/warp_instructions_per_pixel.txt), scaled to this "
                                   "launch's pixels"}  # fmt: skip


def gpu_id(dev: torch.device) -> str:
    """nvidia-smi id of a torch device (its UUID, valid under CUDA_VISIBLE_DEVICES too)."""
    try:
        return "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:  # noqa: BLE001
        return str(dev.index or 0)


def peaks() -> tuple[float, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        return float(json.loads(path.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


REF_DIR = ROOT / "baseline" / "_ref"


def reference_package(backend: str):
    """The unmodified reference package installed under ``baseline/_ref`` with ``backend``
    selected ("reference": its PyTorch CPU backend; "triton": its GPU backend), or None when it
    is not installed there."""
    if not (REF_DIR / "diffrast" / "__init__.py").exists():
        return None
    if str(REF_DIR) not in sys.path:
        sys.path.insert(0, str(REF_DIR))
    import diffrast

    diffrast.set_backend(backend)
    return diffrast


class CpuPath:
    """The render path on the host: the reference package's CPU backend when installed
    (``kind`` "reference"), else the CPU restatement in ``oracle/`` (``kind`` "port")."""

    def __init__(self) -> None:
        self.ref = reference_package("reference")
        self.kind = "reference" if self.ref is not None else "port"
        if self.ref is not None:
            self.ctx = self.ref.RasterizeContext("cpu")
        else:
            import oracle

            self.oracle = oracle

    def rasterize(self, pos, tri, res):
        if self.ref is not None:
            return self.ref.rasterize(self.ctx, pos, tri, res)
        return self.oracle.rasterize(pos, tri, res)

    def interpolate(self, attr, rast, tri, rast_db=None):
        if self.ref is not None:
            if rast_db is None:
                return self.ref.interpolate(attr, rast, tri)
            return self.ref.interpolate(attr, rast, tri, rast_db=rast_db, diff_attrs="all")
        diff = [] if rast_db is None else list(range(attr.shape[-1]))
        return self.oracle.interpolate(attr, rast, tri, rast_db, diff)

    def texture(self, tex, uv, uv_da, mode):
        if self.ref is not None:
            return self.ref.texture(tex, uv, uv_da, filter_mode=mode)
        return self.oracle.texture(tex, uv.contiguous(), None if uv_da is None else uv_da.contiguous(),
                                   None, None, mode, "wrap")

    def antialias(self, color, rast, pos, tri):
        if self.ref is not None:
            return self.ref.antialias(color, rast, pos, tri)
        return self.oracle.antialias(color, rast, pos, tri)

    def describe(self) -> str:
        if self.ref is not None:
            return "the reference package's PyTorch CPU backend (unmodified, baseline/_ref)"
        return "the golden-pinned CPU restatement of the reference backend (oracle/)"


def build_scene(views_total: int, res: int, subdiv: int, tex_size: int, rank: int, world: int):
    import scenes

    from diffrast_b200.distributed import view_shard

    sc = scenes.config5_scene(views=views_total, resolution=res, subdivisions=subdiv, tex_size=tex_size)
    shard = view_shard(views_total, rank, world)
    mvp = sc["mvp"][shard].contiguous()
    gen = torch.Generator().manual_seed(1234)
    target = torch.rand(views_total, res, res, TEX_CHANNELS, generator=gen)[shard]
    return sc["world"].contiguous(), mvp, sc["tri"], sc["attr"], sc["tex"], target.contiguous()


def run_ours(args) -> None:
    import diffrast_b200 as dr
    from diffrast_b200 import _kernels as K
    from diffrast_b200.distributed import NextStepGradientSum, OverlappedGradientSum

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    # All work, eager and captured, runs on one non-default stream, so that the gradient
    # accumulators autograd keeps between steps belong to the stream the graphs capture on.
    work = torch.cuda.Stream(dev)
    torch.cuda.set_stream(work)
    if world > 1:
        from diffrast_b200.distributed import init_process_group

        init_process_group(dev, timeout_s=300)
    if args.views % world:
        raise SystemExit(f"--views {args.views} must be divisible by the number of GPUs {world}")

    world_cpu, mvp_cpu, tri_cpu, attr_cpu, tex_cpu, target_cpu = build_scene(
        args.views, args.res, args.subdiv, args.tex, rank, world)
    views, res = mvp_cpu.shape[0], args.res
    ctx = dr.RasterizeContext(dev)
    tri = tri_cpu.to(dev)
    attr = attr_cpu.to(dev)
    tex = tex_cpu.to(dev).requires_grad_(True)
    verts = world_cpu.to(dev).requires_grad_(True)
    mvp = mvp_cpu.to(dev)
    target = target_cpu.to(dev)
    topo = dr.antialias_construct_topology_hash(tri)
    # On several GPUs the texture gradient's all-reduce runs during the next step's transform,
    # rasterization and interpolation, which do not read the texture, and completes before its
    # lookup (where an optimizer would apply it): synchronous data parallelism with the sum moved
    # from the end of one step to the start of the next (the last step's sum runs after the timed
    # steps, inside the timed region). The positions' all-reduce follows the transform's backward
    # at the end of the step. On one GPU both are no-ops.
    tex_sum = NextStepGradientSum(tex) if world > 1 else None
    reducer = OverlappedGradientSum([verts] if world > 1 else [tex, verts], split_lookups=False)

    def waited(wait):
        if comm_events is None:
            wait()
            return
        # Exposed communication: how long the compute stream waits for the sums.
        before, after = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        before.record()
        wait()
        after.record()
        comm_events.append((before, after))

    def step(mvp_in, target_in, before_loss=None):
        if tex_sum is not None:
            tex_sum.start()
        verts.grad = None
        tex.grad = None
        pos = dr.to_clip(verts, mvp_in)
        rast, rast_db = dr.rasterize(ctx, pos, tri, (res, res))
        out, out_da = dr.interpolate(attr, rast, tri, rast_db=rast_db, diff_attrs="all")
        if tex_sum is not None:
            waited(tex_sum.wait)
        color = dr.texture(tex, out[..., 0:2], out_da[..., 0:4], filter_mode="linear-mipmap-linear")
        # Antialias and the MSE against the target in one pass (dr.antialias_mse fuses the loss
        # into the antialias kernels); the mean runs over the whole job's pixels, so that the
        # ranks' gradients sum to the full batch's.
        if before_loss is not None:
            before_loss()
        _, loss = dr.antialias_mse(color, rast, pos, tri, target_in, topology_hash=topo,
                                   scale=1.0 / (args.views * res * res * TEX_CHANNELS))
        loss.backward()
        waited(reducer.wait)
        if tex_sum is not None:
            tex_sum.hold()
        return loss

    def last_sum():
        """The last step's texture sum (inside the timed region)."""
        if tex_sum is not None:
            tex_sum.start()
            waited(tex_sum.wait)

    comm_events = None

    for _ in range(args.warmup):
        step(mvp, target)
    torch.cuda.synchronize()

    def timed_loop(body):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(args.steps):
            body()
        last_sum()
        end.record()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        ms = torch.tensor([start.elapsed_time(end)], device=dev)
        if world > 1:
            dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        return ms.item() / args.steps

    # Stage times: CUDA events around every launch of an eagerly launched timed pass (a kernel
    # runs the same whether Python or a graph launches it).
    with ClockSampler(gpu_id(dev)) as clocks:
        comm_events = [] if world > 1 else None
        with K.record_timings() as stages:
            ms_eager = timed_loop(lambda: step(mvp, target))
        torch.cuda.synchronize()
    exposed = [b.elapsed_time(a) for b, a in comm_events] if comm_events else []
    comm_events = None
    exposed_ms = torch.tensor([sum(exposed) / args.steps], device=dev)
    if world > 1:
        dist.all_reduce(exposed_ms, op=dist.ReduceOp.MAX)
    stage_ms = {name: sum(s.elapsed_time(e) for s, e in pairs) / args.steps for name, pairs in stages.items()}
    stage_calls = {name: len(pairs) / args.steps for name, pairs in stages.items()}

    # Each step then replays a CUDA graph of the whole forward and backward pass, the gradient
    # all-reduces included: no op reads anything back to the host, so the step captures as a
    # unit. A graph is bound to its input buffers, so each input buffer gets its own (each with its
    # own memory pool). The graphs are released before the process group is destroyed.
    use_graph = not args.eager
    runners: dict[int, object] = {}
    graphs: list = []
    launch_note = "CUDA graph of the step" if use_graph else "eager"

    def runner(mvp_in, target_in):
        if not use_graph:
            return lambda: step(mvp_in, target_in)
        key = mvp_in.data_ptr()
        if key not in runners:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=work):
                loss = step(mvp_in, target_in)
            graphs.append(graph)
            runners[key] = lambda: (graph.replay(), loss)[1]
        return runners[key]

    ms = ms_eager
    if use_graph:
        try:
            run_resident = runner(mvp, target)
        except RuntimeError as exc:  # every rank captures the same step, so all fall back alike
            print(f"bench.py: CUDA graph capture failed, launching eagerly: {exc}", file=sys.stderr)
            use_graph = False
            launch_note = "eager (graph capture failed)"
            torch.cuda.synchronize()
    if use_graph:
        run_resident()
        torch.cuda.synchronize()
        with ClockSampler(gpu_id(dev)) as graph_clocks:
            ms = timed_loop(run_resident)
        clocks = graph_clocks

    # End to end through the public API: every step's inputs are copied from pinned host memory
    # and its loss is read back, all inside the timed region. As an input pipeline would, the copy
    # of step i + 1's inputs runs on a side stream (into the other of two device buffers) while
    # step i computes; the first step's copy is not overlapped.
    mvp_host = mvp_cpu.pin_memory()
    target_host = target_cpu.pin_memory()
    buffers = [(torch.empty_like(mvp_cpu, device=dev), torch.empty_like(target_cpu, device=dev))
               for _ in range(2)]
    for slot in range(2):  # capture (or warm up) outside the timed region
        buffers[slot][0].copy_(mvp)
        buffers[slot][1].copy_(target)
        runner(*buffers[slot])()
    slot_runs = [runner(*buffers[slot]) for slot in range(2)]
    # Warm-up of the host-to-device path itself: the first copies from freshly pinned memory are
    # slower than the steady state.
    for _ in range(2):
        for slot in range(2):
            buffers[slot][0].copy_(mvp_host, non_blocking=True)
            buffers[slot][1].copy_(target_host, non_blocking=True)
    torch.cuda.synchronize()
    copy_stream = torch.cuda.Stream(dev)
    ready = [torch.cuda.Event() for _ in range(2)]
    free = [torch.cuda.Event() for _ in range(2)]

    def upload(slot):
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(free[slot])  # the step that last read this buffer is done
            buffers[slot][0].copy_(mvp_host, non_blocking=True)
            buffers[slot][1].copy_(target_host, non_blocking=True)
            ready[slot].record(copy_stream)

    target_ready = torch.cuda.Event()

    def e2e_loop():
        main = torch.cuda.current_stream(dev)
        for slot in range(2):
            free[slot].record(main)
        # The first step's target is needed only by the antialias pass, so its copy overlaps the
        # step's first kernels (the matrices, 4 KB, go first); that step launches eagerly to wait
        # for it there. Later steps' inputs arrive during the step before.
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(free[0])
            buffers[0][0].copy_(mvp_host, non_blocking=True)
            ready[0].record(copy_stream)
            buffers[0][1].copy_(target_host, non_blocking=True)
            target_ready.record(copy_stream)
        for i in range(args.steps):
            slot = i % 2
            main.wait_event(ready[slot])
            if i + 1 < args.steps:
                upload(1 - slot)
            if i == 0:
                loss = step(*buffers[0], before_loss=lambda: main.wait_event(target_ready))
            else:
                loss = slot_runs[slot]()
            free[slot].record(main)
            loss.item()

    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e2e_start, e2e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2e_start.record()
    e2e_loop()
    last_sum()
    e2e_end.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e2e_t = torch.tensor([e2e_start.elapsed_time(e2e_end)], device=dev)
    if world > 1:
        dist.all_reduce(e2e_t, op=dist.ReduceOp.MAX)
    e2e_ms = e2e_t.item() / args.steps

    # A captured visibility pass that outgrew its binning capacity would have dropped triangles.
    overflow = torch.tensor([1.0 if ctx.capture_overflowed() else 0.0], device=dev)
    if world > 1:
        dist.all_reduce(overflow, op=dist.ReduceOp.MAX)
    if overflow.item():
        raise SystemExit("a captured visibility pass outgrew its binning capacity; rerun")

    pixels_total = args.views * res * res
    value = pixels_total / (ms / 1e3) / 1e6
    e2e_value = pixels_total / (e2e_ms / 1e3) / 1e6
    torch.cuda.synchronize()
    runners.clear()
    for graph in graphs:
        graph.reset()
    graphs.clear()
    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return

    tex_bytes = tex.numel() * 4
    stack_bytes = int(tex_bytes * 4 / 3)
    pixels = views * res * res
    num_vert = verts.shape[0]
    fused = 0 if "interpolate_bwd" in stage_ms else (1 if "resolve_bwd" in stage_ms else 2)
    algo = stage_bytes(pixels, num_vert, views, stack_bytes - tex_bytes, tex_bytes, fused=fused)
    dominant = max(stage_ms, key=stage_ms.get)
    per_launch_ms = stage_ms[dominant] / max(1.0, stage_calls[dominant])
    # Stages launched several times per step (one mip level per launch) are costed per step.
    per_launch_bytes = algo.get(dominant, 0) / max(1.0, stage_calls[dominant])
    peak, peak_kind = peaks()
    achieved = per_launch_bytes / (per_launch_ms / 1e3) / 1e9
    per_call = dict(LAUNCHES)
    per_call["mip_build"], per_call["mip_adjoint"] = mip_launches(args.tex, args.tex, TEX_CHANNELS)
    launches = sum(per_call.get(n, 1) * c for n, c in stage_calls.items())
    clock = clocks.summary()
    line = {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 3),
        "ms_per_step_eager": round(ms_eager, 3),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded icosphere-8, random orbit cameras, uniform texture and target)",
        "config": {
            "workload": f"BASELINE config 5: {args.views} views {res}x{res}, icosphere-{args.subdiv} "
                        f"({tri.shape[0]} tris), tex {args.tex}^2x3 linear-mipmap-linear, antialias, "
                        "MSE, fwd+bwd to tex and pos",
            "views": args.views, "resolution": res, "triangles": int(tri.shape[0]),
            "vertices": num_vert, "tex": args.tex, "parallelism": f"views sharded dp{world}",
            "launch": launch_note,
            "inputs": "per step: the views' 4x4 camera matrices and target images; mesh (world "
                      "positions) and texture are parameters resident on the GPU",
            "l2": "working set larger than L2 (clip positions 671 MB, rast 1 GB per step), no flush",
        },
        "e2e": {"value": round(e2e_value, 1), "unit": UNIT,
                "h2d_bytes_per_step": mvp_cpu.numel() * 4 + target_cpu.numel() * 4,
                "d2h_bytes_per_step": 4},
        "gpu_launches": int(round(launches * args.steps)),
        "roofline": {
            "bound": "hbm", "kernel": dominant, "achieved": round(achieved, 1), "peak": peak,
            "peak_kind": peak_kind, "unit": "GB/s", "frac": round(achieved / peak, 4),
            "traffic": measured_traffic(dominant, pixels),
            "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum per pixel on the "
                              "8-view case, scaled to this launch's pixels",
            "algorithmic_bytes_per_launch": int(per_launch_bytes),
            "ms_per_launch": round(per_launch_ms, 4),
        },
        "issue_roofline": issue_roofline(dominant, pixels, per_launch_ms, clock, dev),
        "step_roofline": {
            "algorithmic_bytes": step_bytes(pixels, num_vert, views, stack_bytes - tex_bytes, tex_bytes),
            "frac_of_peak": round(step_bytes(pixels, num_vert, views, stack_bytes - tex_bytes,
                                             tex_bytes) / (ms / 1e3) / 1e9 / peak, 4),
        },
        "stages_ms": {k: round(v, 3) for k, v in sorted(stage_ms.items(), key=lambda kv: -kv[1])},
        "comm": {
            "allreduce_bytes_per_step": (tex.numel() + verts.numel()) * 4 if world > 1 else 0,
            "exposed_ms_per_step": round(exposed_ms.item(), 3),
            "how": "eager timing pass: CUDA events on the compute stream around its waits for the "
                   "gradient all-reduces (the texture's, run during the next step's transform, "
                   "rasterization and interpolation, waited before its lookup; the positions', at "
                   "the end of the step), per step, max over ranks",
        },
        "clocks": clock,
    }
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args, warmup=1, steps=1)
    if world == 1 and not args.no_gpu_reference:
        # A same-configuration pair: BASELINE configuration 1 in full, this library on the GPU
        # against the reference's CPU backend on the host cores.
        line["config1"] = {
            "workload": "BASELINE config 1: 1 view 256x256, icosphere-3 (1280 tris), tex 256^2x3 "
                        "linear, antialias, MSE, fwd+bwd to tex and pos",
            "gpu": config1_gpu(dev), "cpu_reference": config1_cpu(), "same_config": True,
        }
        # The reference's own GPU backend on this workload (and on config 1), in its own process.
        torch.cuda.empty_cache()
        gpu_ref = gpu_reference_line(args)
        if "config1" in gpu_ref:
            line["config1"]["triton"] = gpu_ref.pop("config1")
        line["gpu_reference"] = gpu_ref
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def cpu_sample(args, path: CpuPath):
    """A bounded CPU sample of the workload: one view of the same scene at a small resolution."""
    world, mvp, tri, attr, tex, _ = build_scene(1, args.cpu_res, args.subdiv, args.tex, 0, 1)
    target = torch.rand(1, args.cpu_res, args.cpu_res, 3, generator=torch.Generator().manual_seed(7))
    res = (args.cpu_res, args.cpu_res)

    def step():
        w = world.clone().requires_grad_(True)
        t = tex.clone().requires_grad_(True)
        # World to clip as diffrast's examples do it (examples/common.py:320-323).
        p = torch.nn.functional.pad(w, (0, 1), value=1.0) @ mvp.transpose(-1, -2)
        rast, rast_db = path.rasterize(p, tri, res)
        out, out_da = path.interpolate(attr, rast, tri, rast_db)
        color = path.texture(t, out[..., 0:2], out_da[..., 0:4], "linear-mipmap-linear")
        image = path.antialias(color, rast, p, tri)
        loss = torch.nn.functional.mse_loss(image, target)
        loss.backward()
        return loss.item()

    return step, res


def cpu_baseline(args, warmup: int, steps: int) -> dict:
    torch.set_num_threads(os.cpu_count() or 1)
    path = CpuPath()
    step, res = cpu_sample(args, path)
    for _ in range(warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    sec = (time.perf_counter() - t0) / steps
    return {
        "value": float(f"{res[0] * res[1] / sec / 1e6:.4g}"),
        "unit": UNIT,
        "cores": torch.get_num_threads(),
        "kind": path.kind,
        "sample": f"1 of {args.views} views of the same scene at {res[0]}x{res[1]} px (full mesh and "
                  f"texture), fwd+bwd, {sec:.2f} s per step, {path.describe()}; the full "
                  "configuration is far beyond the reference CPU backend's brute-force visibility "
                  "(its own benchmark skips it above 2e10 triangle-pixels; this one is 8.8e16)",
    }


def config1_cpu(steps: int = 2, warmup: int = 1) -> dict:
    """BASELINE configuration 1 in full on the host: the reference's CPU backend, all threads."""
    import scenes

    torch.set_num_threads(os.cpu_count() or 1)
    path = CpuPath()
    sc = scenes.config1_scene(seed=0)
    res = sc["resolution"]

    def step():
        pos = sc["pos"].clone().requires_grad_(True)
        tex = sc["tex"].clone().requires_grad_(True)
        rast, _ = path.rasterize(pos, sc["tri"], res)
        uv, _ = path.interpolate(sc["uv"], rast, sc["tri"])
        color = path.texture(tex, uv, None, "linear")
        image = path.antialias(color, rast, pos, sc["tri"])
        torch.nn.functional.mse_loss(image, sc["target"]).backward()

    for _ in range(warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    sec = (time.perf_counter() - t0) / steps
    return {"value": float(f"{res[0] * res[1] / sec / 1e6:.4g}"), "unit": UNIT,
            "ms_per_step": round(sec * 1e3, 1), "cores": torch.get_num_threads(),
            "kind": path.kind, "impl": path.describe()}  # fmt: skip


def config1_gpu(dev: torch.device, steps: int = 200) -> dict:
    """BASELINE configuration 1 in full on one GPU through this library: rasterize, interpolate,
    texture ('linear'), antialias with the fused MSE, backward to texture and positions; each step
    a replay of a CUDA graph of the step, timed with CUDA events."""
    import scenes

    import diffrast_b200 as dr

    sc = scenes.config1_scene(seed=0)
    res = sc["resolution"]
    ctx = dr.RasterizeContext(dev)
    pos = sc["pos"].to(dev).requires_grad_(True)
    tex = sc["tex"].to(dev).requires_grad_(True)
    tri, uv, target = sc["tri"].to(dev), sc["uv"].to(dev), sc["target"].to(dev)

    def step():
        pos.grad = None
        tex.grad = None
        rast, _ = dr.rasterize(ctx, pos, tri, res)
        uvp, _ = dr.interpolate(uv, rast, tri)
        color = dr.texture(tex, uvp, filter_mode="linear")
        _, loss = dr.antialias_mse(color, rast, pos, tri, target)
        loss.backward()
        return loss

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=torch.cuda.current_stream(dev)):
        step()
    for _ in range(10):
        graph.replay()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        graph.replay()
    end.record()
    torch.cuda.synchronize()
    ms = start.elapsed_time(end) / steps
    overflowed = ctx.capture_overflowed()
    graph.reset()
    if overflowed:
        raise SystemExit("config 1: a captured visibility pass outgrew its binning capacity")
    return {"value": round(res[0] * res[1] / (ms / 1e3) / 1e6, 1), "unit": UNIT,
            "ms_per_step": round(ms, 4), "steps": steps, "launch": "CUDA graph of the step"}


def gpu_reference_line(args) -> dict:
    """``bench.py --impl triton`` on the same workload, run in a subprocess (its own CUDA context
    and Triton compilation), or why it could not run."""
    cmd = [sys.executable, str(Path(__file__).resolve()), "--impl", "triton", "--steps",
           str(args.triton_steps), "--warmup", "2", "--views", str(args.views), "--res",
           str(args.res), "--subdiv", str(args.subdiv), "--tex", str(args.tex)]
    env = {k: v for k, v in os.environ.items() if k not in ("RANK", "WORLD_SIZE", "LOCAL_RANK")}
    try:
        done = subprocess.run(cmd, capture_output=True, text=True, timeout=900, env=env)
    except subprocess.TimeoutExpired:
        return {"impl": "triton", "unavailable": "timed out after 900 s"}
    for row in reversed(done.stdout.splitlines()):
        if row.startswith("{"):
            return json.loads(row)
    tail = (done.stderr or done.stdout).strip().splitlines()[-1:] or ["no output"]
    return {"impl": "triton", "unavailable": f"exit {done.returncode}: {tail[0][:300]}"}


def run_triton(args) -> None:
    """The reference's own GPU backend (Triton, unmodified, from baseline/_ref) on the same
    workload and step as this library's arm, on one GPU (rank 0 only)."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    if not torch.cuda.is_available():
        print(json.dumps({"impl": "triton", "unavailable": "no CUDA device"}), flush=True)
        return
    ref = reference_package("triton")
    if ref is None:
        print(json.dumps({"impl": "triton", "unavailable": "the reference package is not installed "
                          "under baseline/_ref"}), flush=True)
        return
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    world_cpu, mvp_cpu, tri_cpu, attr_cpu, tex_cpu, target_cpu = build_scene(
        args.views, args.res, args.subdiv, args.tex, 0, 1)
    res = args.res
    ctx = ref.RasterizeContext(dev)
    tri, attr, mvp, target = (t.to(dev) for t in (tri_cpu, attr_cpu, mvp_cpu, target_cpu))
    tex = tex_cpu.to(dev).requires_grad_(True)
    verts = world_cpu.to(dev).requires_grad_(True)

    def step():
        verts.grad = None
        tex.grad = None
        # World to clip as diffrast's examples do it (examples/common.py:320-323).
        pos = torch.nn.functional.pad(verts, (0, 1), value=1.0) @ mvp.transpose(-1, -2)
        rast, rast_db = ref.rasterize(ctx, pos, tri, (res, res))
        out, out_da = ref.interpolate(attr, rast, tri, rast_db=rast_db, diff_attrs="all")
        color = ref.texture(tex, out[..., 0:2], out_da[..., 0:4], filter_mode="linear-mipmap-linear")
        image = ref.antialias(color, rast, pos, tri)
        loss = torch.nn.functional.mse_loss(image, target)
        loss.backward()
        return loss

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    with ClockSampler(gpu_id(dev)) as clocks:
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(args.steps):
            step()
        end.record()
        torch.cuda.synchronize()
    ms = start.elapsed_time(end) / args.steps
    import triton

    line = {
        "impl": "triton", "metric": METRIC, "value": round(args.views * res * res / (ms / 1e3) / 1e6, 1),
        "unit": UNIT, "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 2), "higher_is_better": True, "dtype": "f32",
        "backend": f"the reference's Triton backend, unmodified (diffrast {ref.__version__}, "
                   f"triton {triton.__version__}), eager launches as the reference runs them",
        "config": {"workload": f"BASELINE config 5: {args.views} views {res}x{res}, "
                               f"icosphere-{args.subdiv}, tex {args.tex}^2x3 linear-mipmap-linear, "
                               "antialias, MSE, fwd+bwd to tex and pos (same as this library's arm)"},
        "peak_mem_gb": round(torch.cuda.max_memory_allocated(dev) / 1e9, 1),
        "clocks": clocks.summary(),
    }  # fmt: skip
    line["config1"] = triton_config1(ref, dev)
    print(json.dumps(line), flush=True)


def triton_config1(ref, dev: torch.device, steps: int = 50) -> dict:
    """BASELINE configuration 1 in full through the reference's Triton backend (the same op
    sequence as config1_gpu, with antialias followed by mse_loss as the reference's API has
    no fused loss), eager as the reference runs it."""
    import scenes

    sc = scenes.config1_scene(seed=0)
    res = sc["resolution"]
    ctx = ref.RasterizeContext(dev)
    pos = sc["pos"].to(dev).requires_grad_(True)
    tex = sc["tex"].to(dev).requires_grad_(True)
    tri, uv, target = sc["tri"].to(dev), sc["uv"].to(dev), sc["target"].to(dev)

    def step():
        pos.grad = None
        tex.grad = None
        rast, _ = ref.rasterize(ctx, pos, tri, res)
        uvp, _ = ref.interpolate(uv, rast, tri)
        color = ref.texture(tex, uvp, filter_mode="linear")
        image = ref.antialias(color, rast, pos, tri)
        torch.nn.functional.mse_loss(image, target).backward()

    for _ in range(5):
        step()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        step()
    end.record()
    torch.cuda.synchronize()
    ms = start.elapsed_time(end) / steps
    return {"value": round(res[0] * res[1] / (ms / 1e3) / 1e6, 1), "unit": UNIT,
            "ms_per_step": round(ms, 3), "steps": steps, "launch": "eager (the reference's API)"}


def run_reference(args) -> None:
    if int(os.environ.get("RANK", "0")) != 0:
        return
    base = cpu_baseline(args, warmup=args.warmup, steps=args.steps)
    line = {
        "metric": METRIC, "value": base["value"], "unit": UNIT, "impl": "reference",
        "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": args.steps,
        "warmup": args.warmup, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic (seeded)",
        "config": {"workload": f"BASELINE config 5 (sample: {base['sample']})"},
        "cpu_baseline": base,
        "e2e": {"value": base["value"], "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }  # fmt: skip
    print(json.dumps(line), flush=True)


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=10)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--impl", choices=["ours", "reference", "triton"], default="ours")
    parser.add_argument("--views", type=int, default=64)
    parser.add_argument("--res", type=int, default=1024)
    parser.add_argument("--subdiv", type=int, default=8)
    parser.add_argument("--tex", type=int, default=4096)
    parser.add_argument("--cpu-res", type=int, default=8)
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--no-gpu-reference", action="store_true",
                        help="skip the reference Triton backend and the config-1 pair")
    parser.add_argument("--triton-steps", type=int, default=5)
    parser.add_argument("--eager", action="store_true",
                        help="launch every step's kernels from Python instead of replaying a CUDA "
                             "graph of the step")
    args = parser.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.impl == "triton":
        run_triton(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
