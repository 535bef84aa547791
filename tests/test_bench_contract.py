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
