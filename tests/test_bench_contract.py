"""The CPU parts of bench.py: the reference arm (the reference's CPU backend, or the oracle port
where the reference package is not installed, on a bounded sample) prints one JSON line with the
keys the benchmark contract asks for; the config-1 CPU timing runs; the Triton arm says why it
cannot run without a GPU."""

import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_reference_arm_prints_one_contract_line():
    out = subprocess.run(
        [sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
         "--warmup", "0", "--cpu-res", "4"],
        cwd=ROOT, capture_output=True, text=True, timeout=600, check=True,
    ).stdout
    lines = [line for line in out.splitlines() if line.startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert line["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["unit"] == "Mpixel/s" and line["value"] > 0
    assert line["cpu_baseline"]["kind"] in ("reference", "port")
    assert line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["value"] == line["value"]


def test_config1_cpu_timing_and_triton_arm_without_gpu():
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "tests"))
    import bench

    c1 = bench.config1_cpu(steps=1, warmup=0)
    assert c1["value"] > 0 and c1["kind"] in ("reference", "port") and c1["cores"] >= 1
    out = subprocess.run(
        [sys.executable, str(ROOT / "bench.py"), "--impl", "triton", "--steps", "1"],
        cwd=ROOT, capture_output=True, text=True, timeout=600, check=True,
    ).stdout
    line = json.loads([row for row in out.splitlines() if row.startswith("{")][-1])
    assert line["impl"] == "triton"
    assert "unavailable" in line or line["value"] > 0


def test_bench_configs_grid_scene_is_the_references():
    """The pipeline-grid scene of bench_configs.py (scenes.displaced_grid) against the reference's
    own benchmark generator's output (tests/golden/bench_grid.npz, made by make_golden.py)."""
    import numpy as np
    import torch

    sys.path.insert(0, str(ROOT / "tests"))
    import scenes

    gold = np.load(ROOT / "tests" / "golden" / "bench_grid.npz")
    pos, tri, uv = scenes.displaced_grid(int(gold["num_tri"]), int(gold["views"]))
    assert torch.equal(tri, torch.from_numpy(gold["tri"]))
    torch.testing.assert_close(pos, torch.from_numpy(gold["pos"]), atol=1e-6, rtol=1e-6)
    assert torch.equal(uv, torch.from_numpy(gold["uv"]))


def test_bench_configs_cases_run_on_the_cpu_path():
    """Every case's op sequence of bench_configs.py, at a small size, through the CPU path that
    bench.py's reference arm uses (the reference package's CPU backend, or the oracle port): the
    steps run and reach the leaves the benchmark differentiates."""
    import torch

    sys.path.insert(0, str(ROOT))
    import bench
    import bench_configs as bc

    ref = bench.reference_package("reference")
    if ref is None:
        import pytest

        pytest.skip("the reference package is not installed under baseline/_ref")
    dev = torch.device("cpu")
    ctx = ref.RasterizeContext(dev)
    cases = [bc.case_c1(dev), bc.case_c2(dev, views=2, size=24, segments=24, sides=6),
             bc.case_c3(dev, views=2, size=24, subdivisions=2, tex_size=16),
             bc.case_c4(dev, views=2, size=24, segments=24, sides=6, cube_size=8),
             bc.case_grid(dev, 200, 24)]
    for name, pixels, what, make in cases:
        fns = make(ref, ctx)
        for fn in fns.values():
            fn()
        assert pixels > 0 and what
        leaves = [t for cell in fns["fwd_bwd"].__closure__ or ()
                  for t in [cell.cell_contents] if isinstance(t, torch.Tensor) and t.requires_grad]
        assert leaves and all(t.grad is not None and t.grad.abs().sum() > 0 for t in leaves), name
