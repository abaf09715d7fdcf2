"""GPU: bench.py's own arm prints one JSON line with every key the driver
reads, on BASELINE config 1 (small, so the run takes seconds): the forward
line (value, roofline, e2e with its copied bytes, clocks, launch count, CPU
baseline, the routing sweep and the same-run parity of the timed inputs) and
the backward line."""
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
REPO = Path(__file__).resolve().parents[1]


def bench_line(*args):
    env = dict(os.environ, WORLD_SIZE="1", RANK="0", LOCAL_RANK="0")
    proc = subprocess.run([sys.executable, str(REPO / "bench.py"), *args], cwd=REPO, env=env,
                          capture_output=True, text=True, timeout=600)
    assert proc.returncode == 0, proc.stderr[-2000:]
    lines = [ln for ln in proc.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, proc.stdout
    return json.loads(lines[0])


def check_common(d, steps, warmup):
    assert d["n_gpus"] == 1 and d["steps"] == steps and d["warmup"] == warmup >= 3
    assert d["value"] > 0 and d["ms_per_step"] > 0 and d["higher_is_better"] is True
    assert d["data"] == "synthetic" and "workload" in d["config"]
    roof = d["roofline"]
    assert roof["achieved"] > 0 and roof["peak"] > 0 and roof["unit"] == "TFLOP/s"
    assert abs(roof["frac"] - roof["achieved"] / roof["peak"]) < 1e-3
    e2e = d["e2e"]
    assert e2e["value"] > 0 and e2e["h2d_bytes_per_step"] > 0 and e2e["d2h_bytes_per_step"] > 0
    assert "sm_mhz" in d["clocks"] and "reasons" in d["clocks"]
    assert d["gpu_launches"] == 2 * steps
    cpu = d["cpu_baseline"]
    assert cpu["value"] > 0 and cpu["cores"] >= 1 and cpu["kind"] in ("reference", "port") and cpu["sample"]
    assert any(p.endswith("libtilemix_b200.so") for p in d["repo_native_so"])


def test_forward_line_on_config1():
    d = bench_line("--config", "c1", "--steps", "2", "--warmup", "3", "--cpu-seconds", "0.2")
    check_common(d, 2, 3)
    sweep = d["routing_sweep"]["points"]
    assert [p["p"] for p in sweep] == [0.0, 0.5, 1.0]
    assert all(p["attention_ms"] > 0 and p["attention_tflops"] > 0 for p in sweep)
    parity = d["parity_of_timed_inputs"]
    assert parity["heads"] == 1 and parity["pass"] and parity["elements_over_max_abs"] == 0


def test_backward_line_on_config1():
    d = bench_line("--op", "backward", "--config", "c1", "--steps", "2", "--warmup", "3", "--cpu-seconds", "0.2")
    check_common(d, 2, 3)
