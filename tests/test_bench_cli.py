"""CPU: bench.py's output contract and constants the attention kernel relies on.

The reference arm runs without a GPU (it times the reference's own CPU path),
so the one-JSON-line-on-stdout contract is checked here; the GPU arm prints
through the same function.
"""
import json
import math
import os
import subprocess
import sys
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parents[1]


def test_reference_arm_prints_exactly_one_json_line():
    env = dict(os.environ, WORLD_SIZE="1", RANK="0", LOCAL_RANK="0")
    proc = subprocess.run([sys.executable, str(REPO / "bench.py"), "--impl", "reference", "--steps", "1",
                           "--warmup", "1", "--cpu-seconds", "0.2"],
                          cwd=REPO, env=env, capture_output=True, text=True, timeout=600)
    assert proc.returncode == 0, proc.stderr[-2000:]
    lines = proc.stdout.splitlines()
    assert len(lines) == 1, proc.stdout
    line = json.loads(lines[0])
    assert line["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    assert line["value"] > 0
    # the reference arm runs the reference's code only: no library of this
    # repository's product is mapped (only oracle/ builds of the reference)
    assert line["repo_native_so"], line
    assert all(p.startswith("oracle/") for p in line["repo_native_so"]), line["repo_native_so"]
    # steps x ms_per_step is time that ran (one bounded sample per step)
    assert line["ms_per_step"] * line["steps"] < 600e3
    assert line["extrapolated_ms_per_full_step"] > 0


def _bench_module():
    import importlib.util
    spec = importlib.util.spec_from_file_location("bench_mod", REPO / "bench.py")
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    return bench


def test_reference_arm_config_is_the_tilemix_arms():
    """Both arms build `config` with the same function from the same arguments,
    so the driver's same-config check holds (outlier note included)."""
    bench = _bench_module()
    env = dict(os.environ, WORLD_SIZE="1", RANK="0", LOCAL_RANK="0")
    proc = subprocess.run([sys.executable, str(REPO / "bench.py"), "--impl", "reference", "--steps", "1",
                           "--warmup", "1", "--cpu-seconds", "0.2"],
                          cwd=REPO, env=env, capture_output=True, text=True, timeout=600)
    assert proc.returncode == 0, proc.stderr[-2000:]
    line = json.loads(proc.stdout.splitlines()[0])
    sys_argv, sys.argv = sys.argv, ["bench.py"]
    try:
        args = bench.parse_args()
    finally:
        sys.argv = sys_argv
    assert line["config"] == bench.config_block(args, 1)
    assert "outlier" in line["config"]["workload"]
    src = (REPO / "bench.py").read_text()
    assert src.count('"config": config_block(args, world)') == 2


def test_reference_arm_under_torchrun_two_ranks_prints_one_line():
    """Under torchrun with two (gloo) ranks, rank 0 alone times and prints; the
    other rank exits 0 without output."""
    env = {k: v for k, v in os.environ.items() if k not in ("WORLD_SIZE", "RANK", "LOCAL_RANK")}
    proc = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
                           "--master-addr", "127.0.0.1", "--master-port", "29547", str(REPO / "bench.py"),
                           "--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "1",
                           "--cpu-seconds", "0.2"],
                          cwd=REPO, env=env, capture_output=True, text=True, timeout=600)
    assert proc.returncode == 0, proc.stderr[-2000:]
    lines = proc.stdout.splitlines()
    assert len(lines) == 1, proc.stdout
    line = json.loads(lines[0])
    assert line["impl"] == "reference" and line["value"] > 0


def test_int8_bias_constants():
    """The attention kernel seeds INT8 accumulators with one f16 MMA of two
    constant tiles: 16 products of fp16 0x6800 and 0x5E00 must sum exactly to
    1.5 * 2^23, whose fp32 bits are 0x4B400000, and a dot |d| < 2^22 added to
    those bits as an integer must read back as the float 1.5 * 2^23 + d."""
    a = np.array([0x6800], np.uint16).view(np.float16)[0]
    b = np.array([0x5E00], np.uint16).view(np.float16)[0]
    assert float(a) == 2048.0 and float(b) == 384.0
    total = np.float32(0)
    for _ in range(16):
        total = np.float32(total + np.float32(a) * np.float32(b))
    assert total == np.float32(1.5 * 2**23)
    assert int(np.array([total], np.float32).view(np.uint32)[0]) == 0x4B400000
    dots = np.array([-(2**22) + 1, -16129 * 128, -1, 0, 1, 16129 * 128, 2**22 - 1], np.int64)
    bits = (0x4B400000 + dots).astype(np.uint32)
    back = bits.view(np.float32).astype(np.float64) - 12582912.0
    assert np.array_equal(back, dots.astype(np.float64))


def test_backward_reference_arm_says_unavailable():
    """The reference is forward only: `--op backward --impl reference` prints
    its one `unavailable` line and exits 0."""
    env = dict(os.environ, WORLD_SIZE="1", RANK="0", LOCAL_RANK="0")
    proc = subprocess.run([sys.executable, str(REPO / "bench.py"), "--op", "backward", "--impl", "reference"],
                          cwd=REPO, env=env, capture_output=True, text=True, timeout=300)
    assert proc.returncode == 0, proc.stderr[-2000:]
    lines = proc.stdout.splitlines()
    assert len(lines) == 1, proc.stdout
    line = json.loads(lines[0])
    assert line["impl"] == "reference" and "backward" in line["unavailable"]


def test_backward_cpu_sample_is_bounded_and_positive():
    bench = _bench_module()
    c = bench.cpu_backward_sample(256, 64, 0.125, True, 0.2)
    assert c["value"] > 0 and c["kind"] == "port" and c["cores"] >= 1


def test_cpu_reference_sample_checks_the_products_output():
    """The CPU-baseline leg compares the sampled heads' reference outputs with
    the output the product computed in the same run: the oracle's own output
    passes, and an output off by 1e-2 in one element fails the 2e-3 bar."""
    import numpy as np
    import oracle
    from tilemix_b200 import workloads
    bench = _bench_module()
    w = workloads.make_inputs("c1", p=0.5, heads=2, seq=128)
    cfg = w["cfg"]
    host = {"q": w["q"].numpy(), "k": w["k"].numpy(), "v": w["v"].numpy(), "words": w["words"].numpy()}
    heads, S, D = w["heads"], w["S"], w["D"]
    wc = host["words"].size // heads
    expect = np.empty((heads, S, D), np.float32)
    for h in range(heads):
        q8, qs = oracle.quantize(host["q"][h], 128)
        k8, ks = oracle.quantize(host["k"][h], 64)
        bits = oracle.decode_routing(host["words"][h * wc:(h + 1) * wc], S, S, 2)[None]
        expect[h] = oracle.tilemix_sampled(host["q"][h:h + 1], host["k"][h:h + 1], host["v"][h:h + 1], q8[None],
                                           k8[None], qs[None], ks[None], bits, np.array([0], np.int32),
                                           np.arange(S, dtype=np.int32), 1.0 / math.sqrt(D), cfg["causal"])[0]
    good = bench.cpu_reference_sample(host, cfg, 100.0, gpu_out=expect)["parity"]
    assert good["heads"] == heads and good["pass"] and good["max_abs"] < 1e-6
    bad_out = expect.copy()
    bad_out[1, 5, 7] += 1e-2
    bad = bench.cpu_reference_sample(host, cfg, 100.0, gpu_out=bad_out)["parity"]
    assert not bad["pass"] and abs(bad["max_abs"] - 1e-2) < 1e-4
