#!/usr/bin/env python
"""TileMix B200 benchmark: effective attention TFLOP/s on a BASELINE config.

One step = the TileMix hot path over one batch: stage-1 INT8 quantization of Q
and K, then the fused routed attention kernel (quantize_tilemix_qk_batched +
tilemix_attention_batched through the C-ABI). Default workload: BASELINE
config 3 (B8 H32 S4096 D128, causal, 1% x20 outlier channels, INT8 routing
Bernoulli(0.75) over 64x64 tiles) -- the configuration the north-star target is
quoted on.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--config c3] [--p P]
  python bench.py --impl reference ...   (the reference's CPU path, rank 0)
  python bench.py --op backward ...      (the unrouted attention's backward on the
                                          config's shapes; no reference counterpart)

Multi-GPU (torchrun, one process per GPU): the batch's B*H heads are split
into contiguous per-rank shards (strong scaling: the job is one config-3 batch
at every N; independent (b, h) heads, no collective on the data path;
--scaling weak gives every rank its own full batch instead). NCCL is used only
for the start/stop barriers and the max-over-ranks reduction of the device
times. Rank 0 prints one JSON line.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from datetime import datetime, timedelta
from pathlib import Path

REPO = Path(__file__).resolve().parent
for p in (REPO, REPO / "tilemix-cuda_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

METRIC = "effective attention TFLOP/s and % of mix-weighted tensor peak, 1/2/4/8 B200"


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="tilemix", choices=["tilemix", "reference"])
    ap.add_argument("--config", default="c3")
    ap.add_argument("--p", type=float, default=None, help="override the INT8 routing fraction")
    ap.add_argument("--cpu-seconds", type=float, default=6.0,
                    help="target CPU time of one reference-arm sample")
    ap.add_argument("--routing", default="mask", choices=["mask", "policy"],
                    help="mask: the config's Bernoulli 64x64 routing mask; policy: routing words chosen on the "
                         "device from the quantizer's block scales each step (tilemix_routing_policy)")
    ap.add_argument("--tau", type=float, default=1.0,
                    help="policy: bound on the INT8 score error (score units) that a tile may incur")
    ap.add_argument("--v-hint", action="store_true",
                    help="quantize_tilemix_qkv_batched records max |v| per 64-key block and the attention takes "
                         "single-term fp16 P where it is <= 3.5 (tilemix_attention_batched_hinted)")
    ap.add_argument("--scaling", default="strong", choices=["weak", "strong"],
                    help="strong (default): the batch's heads are split over ranks; weak: every rank runs a full batch")
    ap.add_argument("--heads", type=int, default=None,
                    help="--op backward only: run this many of the config's B*H heads (small profiling captures)")
    ap.add_argument("--op", default="attention", choices=["attention", "backward"],
                    help="attention (default): the routed forward hot path; backward: dQ, dK, dV of the unrouted "
                         "attention (tilemix_attention_backward on the training forward's row LSE)")
    return ap.parse_args()


def measured_peaks() -> dict:
    path = REPO / "MEASURED_PEAKS.json"
    if path.exists():
        d = json.loads(path.read_text())
        return {"bf16_tflops": d["bf16_tflops"], "bf16_tflops_sustained": d["bf16_tflops_sustained"],
                "hbm_gbs": d["hbm_gbs"], "source": "measured"}
    return {"bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "hbm_gbs": 6650.0, "source": "fallback"}


def measured_int8_tops() -> float | None:
    """Measured dense INT8 GEMM throughput from the committed profile summary
    (MEASURED_PEAKS.json holds no INT8 figure)."""
    for path in sorted((REPO / "profiles").glob("*.txt")):
        for line in path.read_text().splitlines():
            if line.startswith("measured_int8_tops "):
                return float(line.split()[1])
    return None


def profiled_traffic() -> dict:
    """ncu DRAM bytes per unit of work for the attention kernel, from the
    committed summary under profiles/ (null when absent)."""
    out = {}
    for path in sorted((REPO / "profiles").glob("*.txt")):
        for line in path.read_text().splitlines():
            if line.startswith("bench_traffic_per_head "):
                _, cfg, value = line.split()
                out[cfg] = float(value)
    return out


# ------------------------------------------------------------------ clocks
class ClockSampler:
    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.proc = None
        self.gpu = gpu_index
        self.window = None       # (start, end) host wall-clock of the timed region

    def mark(self, start: float, end: float):
        self.window = (start, end)

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "20"],
                stdout=self.file, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.flush()
        rows = []
        with open(self.file.name) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) < 10:
                    continue
                try:
                    stamp = datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                except ValueError:
                    continue
                # keep the samples taken while the timed region ran
                if self.window is None or self.window[0] <= stamp <= self.window[1]:
                    rows.append(parts[1:])
        os.unlink(self.file.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        smax = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        power = [float(r[3]) for r in rows if r[3].replace(".", "").isdigit()]
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": reasons, "samples": len(rows),
                "power_w_max": max(power) if power else None}


# ------------------------------------------------------------------ output
_JSON_OUT = None


def claim_stdout() -> None:
    """Keep the process's stdout for the one JSON line and point file
    descriptor 1 at stderr, so nothing a library prints on its own (NCCL's
    version banner on hosts that set NCCL_DEBUG, for one) can reach stdout."""
    global _JSON_OUT
    sys.stdout.flush()
    _JSON_OUT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)


def emit(line: dict) -> None:
    out = _JSON_OUT if _JSON_OUT is not None else sys.stdout
    out.write(json.dumps(line) + "\n")
    out.flush()


# -------------------------------------------------------------- distributed
def dist_setup(args):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    # Keep stdout to the one JSON line: NCCL writes its log (and, at
    # NCCL_DEBUG=WARN or VERSION, a version banner) to stdout unless
    # NCCL_DEBUG_FILE names another file.
    os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
    if world > 1:
        import torch.distributed as dist
        if args.impl == "tilemix":
            torch.cuda.set_device(local)
            dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                    device_id=torch.device(f"cuda:{local}"))
        else:
            dist.init_process_group("gloo", timeout=timedelta(seconds=300))
    elif args.impl == "tilemix":
        torch.cuda.set_device(local)
    return rank, world, local


def reduce_max(value: float, world: int) -> float:
    from tilemix_b200 import sharding
    return sharding.max_over_ranks(value, world, device="cuda")


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def repo_libraries() -> list[str]:
    """Shared objects under this repository mapped into this process (from
    /proc/self/maps): which native code an arm actually ran."""
    found = set()
    try:
        with open("/proc/self/maps") as f:
            for line in f:
                path = line.split()[-1] if len(line.split()) >= 6 else ""
                if path.startswith(str(REPO)) and ".so" in Path(path).name:
                    found.add(str(Path(path).relative_to(REPO)))
    except OSError:
        pass
    return sorted(found)


# ------------------------------------------------------------------ config
def config_block(args, world: int) -> dict:
    """The `config` object of the JSON line; both arms print it identically."""
    from tilemix_b200 import workloads
    cfg = workloads.config(args.config, p=args.p)
    routing = (f"INT8 routing by the device policy (tau={args.tau})" if args.routing == "policy"
               else f"INT8 routing p={cfg['p']}")
    if args.v_hint:
        routing += ", single-term P where max|v| <= 3.5"
    label = (f"{args.config}: B{cfg['B']} H{cfg['H']} S{cfg['S']} D{cfg['D']}"
             f"{' causal' if cfg['causal'] else ''}, {routing}"
             f"{', x20 outlier channels' if cfg['outliers'] else ''}")
    split = ("heads split into contiguous per-rank shards" if args.scaling == "strong"
             else "every rank runs its own full batch")
    return {"workload": label, "B": cfg["B"], "H": cfg["H"], "S": cfg["S"], "D": cfg["D"],
            "causal": cfg["causal"], "int8_fraction_requested": cfg["p"],
            "parallelism": f"batch x head shards over {world} GPU rank(s) ({args.scaling}: {split}), no collective",
            "l2": "inputs larger than L2 (126 MiB) at the default configs; no flush"}


# ------------------------------------------------------------- CPU baseline
def cpu_reference_sample(w_host: dict, cfg: dict, target_s: float, gpu_out=None) -> dict:
    """Time the reference's own CPU path (oracle/_ref: reference_quantize and
    reference_tilemix from src/tests/reference_tilemix.h; a causal row runs the
    reference on its key prefix) on a bounded sample of the workload -- whole
    heads, all rows, on all host cores -- and extrapolate to the full batch.
    Falls back to the C restatement (kind "port") without the reference build.
    With gpu_out ([heads, S, D] fp32 on the host: what the product computed
    from the same inputs in this run), the sampled heads' reference outputs
    are also compared with it (the checker, not part of the timed product)."""
    import numpy as np
    import oracle
    if not oracle.ORACLE_SO.exists() or (not oracle.ref_available() and oracle.reference_tree_present()):
        oracle.build()
    kind = "reference" if oracle.ref_available() else "port"
    use_ref = kind == "reference"
    # every host core this process may use (torchrun sets OMP_NUM_THREADS=1)
    oracle.set_threads(len(os.sched_getaffinity(0)))
    q, k, v = w_host["q"], w_host["k"], w_host["v"]
    avail, S, D = q.shape
    H = cfg["B"] * cfg["H"]            # heads of the whole workload
    causal = cfg["causal"]
    wc = w_host["words"].size // avail
    rows = np.arange(S, dtype=np.int32)
    keys = np.minimum(rows + 1, S) if causal else np.full(S, S)
    head_flops = float((4.0 * keys * D).sum())
    threads = oracle.ref_lib().ref_max_threads() if use_ref else oracle.max_threads()

    def run_head(h):
        sl = slice(h, h + 1)
        t = time.perf_counter()
        if use_ref:
            q8, qs = oracle.ref_quantize(q[h], 128)
            k8, ks = oracle.ref_quantize(k[h], 64)
        else:
            q8, qs = oracle.quantize(q[h], 128)
            k8, ks = oracle.quantize(k[h], 64)
        t_quant = time.perf_counter() - t
        bits = oracle.decode_routing(w_host["words"][h * wc:(h + 1) * wc], S, S, 2)[None]
        t = time.perf_counter()
        ref = oracle.tilemix_sampled(q[sl], k[sl], v[sl], q8[None], k8[None], qs[None], ks[None], bits,
                                     np.array([0], np.int32), rows, 1.0 / math.sqrt(D), causal,
                                     use_reference=use_ref)
        elapsed = time.perf_counter() - t
        if gpu_out is not None:
            diff = np.abs(gpu_out[h].astype(np.float64) - ref[0])
            checks.append((float(diff.max()), float(np.sum(diff * diff)), float(np.sum(ref[0] * ref[0])),
                           int(np.count_nonzero(diff > 2e-3)), int(diff.size)))
        return t_quant, elapsed

    checks = []
    tq, ta = run_head(0)
    n_heads = int(max(1, min(avail, math.ceil(target_s / max(ta + tq, 1e-6)))))
    for h in range(1, n_heads):
        a, b = run_head(h)
        tq += a
        ta += b
    rate = n_heads * head_flops / ta                       # attention FLOP/s on all threads
    quant_per_head = tq / n_heads                          # seconds, one thread
    from tilemix_b200 import workloads
    f_eff = workloads.effective_flops(cfg)
    step_s = f_eff / rate + quant_per_head * H / threads   # quantization parallel over heads
    result = {"value": f_eff / step_s / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": kind,
              "sample": (f"{n_heads} whole head(s) of S={S} through reference_quantize (1 thread) and "
                         f"reference_tilemix ({'causal: each row on its key prefix, ' if causal else ''}"
                         f"{threads} OpenMP threads over rows; {ta + tq:.1f} s), extrapolated to all {H} heads"),
              "step_seconds": step_s}
    if checks:
        max_abs = max(c[0] for c in checks)
        rel_l2 = math.sqrt(sum(c[1] for c in checks) / max(sum(c[2] for c in checks), 1e-300))
        result["parity"] = {"heads": len(checks), "max_abs": max_abs, "rel_l2": rel_l2,
                            "bar": "max_abs <= 2e-3 and rel_l2 <= 1e-3",
                            "pass": bool(max_abs <= 2e-3 and rel_l2 <= 1e-3),
                            "elements_over_max_abs": sum(c[3] for c in checks),
                            "elements": sum(c[4] for c in checks),
                            "against": f"reference_tilemix ({kind}) on this run's inputs and routing words; the "
                                       "product's output from the end-to-end leg",
                            "note": "errors concentrate on the x20 outlier channels, where FP16 scores q.k reach "
                                    "thousands and the tensor core's fp32 accumulation of the fp16 products "
                                    "limits them; the reference's own WMMA kernel has the same error profile on "
                                    "such inputs (tests/test_gpu_reference_kernel.py)"}
    return result


# ------------------------------------------------------------------ our arm
def run_tilemix(args, rank, world, local):
    import numpy as np
    import torch
    import tilemix_b200 as tm
    from tilemix_b200 import workloads

    from tilemix_b200 import sharding
    cfg0 = workloads.config(args.config, p=args.p)
    total_heads = cfg0["B"] * cfg0["H"]
    if args.scaling == "strong":
        _, my_heads = sharding.shard_heads(total_heads, world, rank)
        w = workloads.make_inputs(args.config, p=args.p, batch=1, heads=my_heads,
                                  seed=sharding.rank_seed(cfg0["seed"], rank), device="cuda")
    else:
        w = workloads.make_inputs(args.config, p=args.p, seed=sharding.rank_seed(cfg0["seed"], rank),
                                  device="cuda")
    cfg, H, S, D = w["cfg"], w["heads"], w["S"], w["D"]
    job_flops = (world * workloads.effective_flops(cfg0) if args.scaling == "weak"
                 else workloads.effective_flops(cfg0))
    q, k, v = w["q"], w["k"], w["v"]
    words = w["words"].cuda()
    q8 = torch.empty_like(q, dtype=torch.int8)
    k8 = torch.empty_like(k, dtype=torch.int8)
    qs = torch.empty((H, (S - 1) // 128 + 1), dtype=torch.float16, device="cuda")
    ks = torch.empty((H, (S - 1) // 64 + 1), dtype=torch.float16, device="cuda")
    out = torch.empty((H, S, D), dtype=torch.float32, device="cuda")
    routing = tm.TileMixRouting(words, words.numel(), 2)
    quantized = tm.TileMixQuantized(q8, k8, qs, ks)
    stream = torch.cuda.current_stream()
    f_eff = workloads.effective_flops(cfg, H)       # this rank's work per step
    f_real = workloads.realised_int8_fraction(w["mask"], cfg["causal"])

    policy = args.routing == "policy"
    max_product = tm.tilemix_policy_max_scale_product(args.tau, w["score_scale"], D) if policy else None

    v_absmax = torch.empty((H, (S - 1) // 64 + 1), dtype=torch.float16, device="cuda") if args.v_hint else None

    def quantize():
        if args.v_hint:
            tm.check(tm.quantize_tilemix_qkv_batched(q, k, v, q8, k8, qs, ks, v_absmax, H, S, S, D, stream), "quantize")
        else:
            tm.check(tm.quantize_tilemix_qk_batched(q, k, q8, k8, qs, ks, H, S, S, D, stream), "quantize")
        if policy:   # routing words from this step's block scales, on the device
            tm.check(tm.tilemix_routing_policy(qs, ks, words, H, S, S, 2, max_product, stream), "routing policy")

    def attend():
        if args.v_hint:
            tm.check(tm.tilemix_attention_batched_hinted(q, k, v, out, H, S, S, D, w["score_scale"], cfg["causal"],
                                                         stream, routing, quantized, v_absmax), "attention")
        else:
            tm.check(tm.tilemix_attention_batched(q, k, v, out, H, S, S, D, w["score_scale"], cfg["causal"],
                                                  stream, routing, quantized), "attention")

    for _ in range(args.warmup):
        quantize(); attend()
    torch.cuda.synchronize()

    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)                     # let the sampler attach before the timed region
    n = args.steps
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2 * n + 2)]
    barrier(world)
    torch.cuda.synchronize()
    t_start = time.time()
    ev[0].record(stream)
    for i in range(n):
        quantize()
        ev[1 + 2 * i].record(stream)
        attend()
        ev[2 + 2 * i].record(stream)
    ev[-1].record(stream)
    torch.cuda.synchronize()
    clocks.mark(t_start, time.time())
    barrier(world)
    clk = clocks.stop()
    total_ms = ev[0].elapsed_time(ev[-1])
    attn_ms = [ev[1 + 2 * i].elapsed_time(ev[2 + 2 * i]) for i in range(n)]
    quant_ms = [(ev[0] if i == 0 else ev[2 * i]).elapsed_time(ev[1 + 2 * i]) for i in range(n)]
    err, status = tm.read_and_clear_status()
    tm.check(err, "status")
    if status:
        raise SystemExit(f"kernel watchdog reported status {status:#x}")
    if policy:
        f_real = workloads.int8_fraction_from_words(words.cpu().numpy(), H, S, cfg["causal"])
    single_share = (float((v_absmax.float() <= 3.5).float().mean()) if args.v_hint else 0.0)
    sweep = (routing_sweep(args, cfg, w, out, quantized, stream, world, job_flops)
             if not policy and not args.v_hint else None)
    step_ms = reduce_max(total_ms / n, world)
    attn_avg = reduce_max(sum(attn_ms) / n, world)
    quant_avg = reduce_max(sum(quant_ms) / n, world)

    # end to end through the C-ABI with host buffers: one
    # tilemix_attention_from_host call per step (H2D of Q, K, V and the
    # routing words, both kernels, D2H of the fp32 output, pipelined over
    # chunks of heads inside the library).
    hq, hk, hv = (t.cpu().pin_memory() for t in (q, k, v))
    hwords = (words.cpu() if policy else w["words"]).pin_memory()   # the words the timed steps used
    hout = torch.empty((H, S, D), dtype=torch.float32).pin_memory()
    bufs = tm.TileMixDeviceBuffers(q=q, k=k, v=v, q8=q8, k8=k8, q_scales=qs, k_scales=ks, words=words, o=out)
    e2e_steps = max(1, min(n, 5))

    def e2e_step():
        tm.check(tm.tilemix_attention_from_host(hq, hk, hv, hwords, hout, bufs, H, S, S, D, w["score_scale"],
                                                cfg["causal"], 2, 0, stream), "attention_from_host")

    e2e_step()
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    e2e_ms = reduce_max(e0.elapsed_time(e1) / e2e_steps, world)
    h2d = 3 * q.numel() * 2 + words.numel() * 8
    d2h = out.numel() * 4

    # Host-link bandwidth with every rank copying at once (what bounds the
    # end-to-end leg): one pinned H2D copy of this rank's Q and one D2H copy
    # of its fp32 O, each timed on the stream; the slowest rank counts.
    def timed_copy(dst, src):
        barrier(world)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        dst.copy_(src, non_blocking=True)
        b.record(stream)
        torch.cuda.synchronize()
        return reduce_max(a.elapsed_time(b), world)
    h2d_ms = timed_copy(q, hq)
    d2h_ms = timed_copy(hout, out)
    link = {"h2d_gbs_per_rank": round(q.numel() * 2 / (h2d_ms * 1e-3) / 1e9, 2),
            "d2h_gbs_per_rank": round(out.numel() * 4 / (d2h_ms * 1e-3) / 1e9, 2),
            "ranks_copying_at_once": world}

    cpu = None
    parity = None
    if rank == 0 and world == 1:
        nh = min(H, 32)
        host = {"q": hq.numpy()[:nh].copy(), "k": hk.numpy()[:nh].copy(), "v": hv.numpy()[:nh].copy(),
                "words": hwords.numpy()[: nh * (hwords.numel() // H)].copy()}
        c = cpu_reference_sample(host, cfg, args.cpu_seconds, gpu_out=hout.numpy()[:nh])
        cpu = {key: c[key] for key in ("value", "unit", "cores", "kind", "sample")}
        parity = c.get("parity")

    if rank != 0:
        return
    peaks = measured_peaks()
    achieved = f_eff / (attn_avg * 1e-3) / 1e12
    traffic_per_head = profiled_traffic().get(args.config)
    value = job_flops / (step_ms * 1e-3) / 1e12
    p_mix = workloads.mix_peak(f_eff, f_real) / 1e12
    i8_meas = measured_int8_tops()
    p_mix_meas = (workloads.mix_peak(f_eff, f_real, p_f16=peaks["bf16_tflops"] * 1e12, p_i8=i8_meas * 1e12) / 1e12
                  if i8_meas else None)
    # The op's own peak: the mix-weighted tensor peak at this launch's realised
    # INT8 share, from the measured bf16 GEMM (burst) and the measured INT8 GEMM.
    if p_mix_meas is not None:
        peak = p_mix_meas
        peak_source = (f"mix-weighted peak at INT8 share {f_real:.3f} of the QK work: {peaks['source']} bf16 dense "
                       f"{peaks['bf16_tflops']} TFLOP/s (burst, MEASURED_PEAKS.json) and measured INT8 GEMM "
                       f"{i8_meas} TOPS (profiles/gemm_peaks_int8_fp16.txt)")
    else:
        peak = peaks["bf16_tflops"]
        peak_source = f"{peaks['source']} bf16 dense (burst), MEASURED_PEAKS.json (no INT8 figure found)"
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world,
        "steps": n, "warmup": args.warmup, "ms_per_step": round(step_ms, 4), "higher_is_better": True,
        "scaling": args.scaling, "vs_baseline": None, "dtype": "f16+i8 (f32 accumulate)", "data": "synthetic",
        "config": config_block(args, world),
        "int8_fraction_realised": round(f_real, 4), "per_gpu_heads": H,
        "inputs_mib_per_gpu": round(3 * q.numel() * 2 / 2**20, 1),
        "pct_of_mix_peak": round(100 * (f_eff / (step_ms * 1e-3) / 1e12) / p_mix, 2),
        "mix_peak_tflops": round(p_mix, 1),
        "mix_peak_basis": "NVIDIA dense figures: 2250 TFLOP/s fp16, 4500 TOPS int8",
        "pct_of_mix_peak_measured": (round(100 * (f_eff / (step_ms * 1e-3) / 1e12) / p_mix_meas, 2)
                                     if p_mix_meas else None),
        "mix_peak_measured_tflops": round(p_mix_meas, 1) if p_mix_meas else None,
        "attention_ms": round(attn_avg, 4), "quantize_ms": round(quant_avg, 4),
        "quantize_gbs": round(3 * 2 * H * S * D / (quant_avg * 1e-3) / 1e9, 1),
        "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": round(peak, 1), "unit": "TFLOP/s",
                     "frac": round(achieved / peak, 4),
                     "peak_source": peak_source,
                     "frac_of_bf16_peak": round(achieved / peaks["bf16_tflops"], 4),
                     "traffic": None if traffic_per_head is None else traffic_per_head * H,
                     "kernel": "tilemix_attention_kernel",
                     "work": "F_eff = 4*B*H*S^2*D/2 (causal) algorithmic FLOPs per launch"},
        "e2e": {"value": round(job_flops / (e2e_ms * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 3),
                "api": "tilemix_attention_from_host (C-ABI, pinned host buffers, pipelined over head chunks)",
                "host_link": link},
        "clocks": clk,
        "gpu_launches": (3 if policy else 2) * n,
        "pv_single_term_share": round(single_share, 4),
        "routing": ({"kind": "policy", "tau": args.tau, "max_scale_product": max_product,
                     "note": "INT8 iff q_scale * max k_scale <= max_scale_product (tilemix_routing_policy, every step)"}
                    if policy else {"kind": "mask", "note": "the config's Bernoulli 64x64 INT8 mask"}),
        "repo_native_so": repo_libraries(),
    }
    if sweep is not None:
        mix = workloads.mix_peak
        for row in sweep:
            meas = (mix(f_eff, row["int8_fraction_realised"], p_f16=peaks["bf16_tflops"] * 1e12,
                        p_i8=i8_meas * 1e12) / 1e12 if i8_meas else None)
            row["pct_of_mix_peak_measured"] = round(100 * row["attention_tflops_per_gpu"] / meas, 2) if meas else None
        line["routing_sweep"] = {
            "note": "attention kernel alone on this run's Q/K/V/Q8/K8, other Bernoulli 64x64 INT8 masks "
                    "(p = 0.5 is the north star's operating point); device-timed, max over ranks; attention_tflops "
                    "job-wide like value, attention_tflops_per_gpu and pct_of_mix_peak_measured per GPU",
            "points": sweep}
    if cpu is not None:
        line["cpu_baseline"] = cpu
    if parity is not None:
        line["parity_of_timed_inputs"] = parity
    emit(line)


def routing_sweep(args, cfg, w, out, quantized, stream, world, job_flops, ps=(0.0, 0.5, 1.0), launches=10):
    """Attention alone at other INT8 routing fractions on the same inputs:
    a fresh Bernoulli 64x64 mask per point (seeded from the config's seed),
    `launches` timed launches after one untimed one; TFLOP/s per GPU (this
    rank's heads) and for the whole job (max time over ranks)."""
    import torch
    import tilemix_b200 as tm
    from tilemix_b200 import workloads
    H, S, D = w["heads"], w["S"], w["D"]
    qb = (S + 63) // 64
    f_eff = workloads.effective_flops(cfg, H)
    points = []
    for i, p in enumerate(ps):
        g = torch.Generator().manual_seed(cfg["seed"] * 1000 + i)
        mask = (torch.rand((H, qb, qb), generator=g) < p).to(torch.uint8)
        words = torch.from_numpy(workloads.pack_block_mask64(mask.numpy(), S, S)).cuda()
        routing = tm.TileMixRouting(words, words.numel(), 2)

        def attend():
            tm.check(tm.tilemix_attention_batched(w["q"], w["k"], w["v"], out, H, S, S, D, w["score_scale"],
                                                  cfg["causal"], stream, routing, quantized), "attention")
        attend()
        barrier(world)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(launches):
            attend()
        b.record(stream)
        torch.cuda.synchronize()
        ms = reduce_max(a.elapsed_time(b) / launches, world)
        points.append({"p": p, "int8_fraction_realised": round(workloads.realised_int8_fraction(mask, cfg["causal"]), 4),
                       "attention_ms": round(ms, 4), "attention_tflops": round(job_flops / (ms * 1e-3) / 1e12, 1),
                       "attention_tflops_per_gpu": round(f_eff / (ms * 1e-3) / 1e12, 1)})
    err, status = tm.read_and_clear_status()
    tm.check(err, "status")
    if status:
        raise SystemExit(f"kernel watchdog reported status {status:#x}")
    return points


# ------------------------------------------------------------ backward arm
def cpu_backward_sample(S: int, D: int, scale: float, causal: bool, target_s: float) -> dict:
    """The same gradient formula in float32 torch autograd on the host cores,
    on whole heads at the config's S and D: the CPU baseline of the backward
    line (the reference has no backward to time)."""
    import torch
    threads = torch.get_num_threads()
    S_cfg, S = S, min(S, 4096)     # the S x S matrices of one head stay a few hundred MB
    g = torch.Generator().manual_seed(7)
    q, k, v, do = (torch.randn((1, S, D), generator=g) for _ in range(4))

    def one():
        qg, kg, vg = (t.clone().requires_grad_() for t in (q, k, v))
        s = scale * qg @ kg.transpose(-1, -2)
        if causal:
            s = s.masked_fill(torch.ones(S, S, dtype=torch.bool).triu(1), float("-inf"))
        o = torch.softmax(s, -1) @ vg
        o.backward(do)
    one()                                  # warm-up: thread pool, allocator
    t0 = time.perf_counter()
    one()
    per_head = time.perf_counter() - t0
    heads = max(1, min(64, int(target_s / max(per_head, 1e-3))))
    t0 = time.perf_counter()
    for _ in range(heads):
        one()
    secs = time.perf_counter() - t0
    flops = 2.5 * 4.0 * heads * S * S * D * (0.5 if causal else 1.0)
    return {"value": round(flops / secs / 1e12, 5), "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"{heads} head(s) of S={S}{f' (the config has S={S_cfg}; TFLOP/s compared per FLOP)' if S != S_cfg else ''}, "
                      f"D={D}{' causal' if causal else ''} through float32 torch autograd "
                      f"of softmax(score_scale q k^T) v on {threads} threads ({secs:.1f} s); the reference has no "
                      f"backward, so this is the formula, not the reference's code"}


def run_backward(args, rank, world, local):
    """dQ, dK, dV of the unrouted attention on the config's shapes: setup runs
    the training forward once (tilemix_attention_batched_lse: O and the row
    LSE); one step = tilemix_attention_backward on that LSE (row kernel: dQ
    and D = rowsum(dO * O); column kernel: dK, dV). Work counted as the five
    gradient products, 10 * S^2 * D per head (2.5x the forward), halved for
    causal."""
    import torch
    import tilemix_b200 as tm
    from tilemix_b200 import sharding, workloads

    cfg0 = workloads.config(args.config)
    if args.heads is not None:
        cfg0 = workloads.config(args.config, B=1, H=args.heads)
    total_heads = cfg0["B"] * cfg0["H"]
    if args.scaling == "strong":
        _, my_heads = sharding.shard_heads(total_heads, world, rank)
    else:
        my_heads = total_heads
    w = workloads.make_inputs(args.config, batch=1, heads=my_heads, seed=sharding.rank_seed(cfg0["seed"], rank),
                              device="cuda")
    cfg, H, S, D = w["cfg"], w["heads"], w["S"], w["D"]
    causal, scale = cfg["causal"], w["score_scale"]
    q, k, v = w["q"], w["k"], w["v"]
    g = torch.Generator(device="cuda").manual_seed(cfg0["seed"] + 101 + rank)
    do = torch.randn((H, S, D), generator=g, device="cuda").half()
    o = torch.empty((H, S, D), dtype=torch.float32, device="cuda")
    dq, dk, dv = (torch.empty((H, S, D), dtype=torch.float32, device="cuda") for _ in range(3))
    lse = torch.empty((H, S), dtype=torch.float32, device="cuda")
    dsum = torch.empty((H, S), dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream()

    def forward():
        tm.check(tm.tilemix_attention_batched_lse(q, k, v, o, lse, H, S, S, D, scale, causal, stream), "forward")

    def backward():
        tm.check(tm.tilemix_attention_backward(q, k, v, o, do, dq, dk, dv, lse, dsum, H, S, S, D, scale, causal,
                                               stream, lse_from_forward=True), "backward")

    forward()
    for _ in range(args.warmup):
        backward()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    n = args.steps
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    t_start = time.time()
    e0.record(stream)
    for _ in range(n):
        backward()
    e1.record(stream)
    torch.cuda.synchronize()
    clocks.mark(t_start, time.time())
    barrier(world)
    clk = clocks.stop()
    step_ms = reduce_max(e0.elapsed_time(e1) / n, world)
    # the forward that produces O and the LSE, timed alone for the training step
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for _ in range(5):
        forward()
    f1.record(stream)
    torch.cuda.synchronize()
    fwd_ms = reduce_max(f0.elapsed_time(f1) / 5, world)
    err, status = tm.read_and_clear_status()
    tm.check(err, "status")
    if status:
        raise SystemExit(f"kernel watchdog reported status {status:#x}")

    # end to end through the C-ABI with host buffers: per step the H2D copies of
    # Q, K, V and dO from pinned memory, the training forward, the backward and
    # the D2H copies of dQ, dK, dV
    hq, hk, hv, hdo = (t.cpu().pin_memory() for t in (q, k, v, do))
    hdq, hdk, hdv = (torch.empty((H, S, D), dtype=torch.float32).pin_memory() for _ in range(3))

    def e2e_step():
        for dst, src in ((q, hq), (k, hk), (v, hv), (do, hdo)):
            dst.copy_(src, non_blocking=True)
        forward()
        backward()
        for dst, src in ((hdq, dq), (hdk, dk), (hdv, dv)):
            dst.copy_(src, non_blocking=True)
    e2e_step()
    torch.cuda.synchronize()
    barrier(world)
    e2e_steps = max(1, min(n, 3))
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    b.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    e2e_ms = reduce_max(a.elapsed_time(b) / e2e_steps, world)

    cpu = None
    if rank == 0 and world == 1:
        cpu = cpu_backward_sample(S, D, scale, causal, args.cpu_seconds)
    if rank != 0:
        return
    peaks = measured_peaks()
    # what one step touches: Q, K, V, dO (fp16), O, dQ, dK, dV (fp32)
    footprint_mib = (4 * q.numel() * 2 + 4 * o.numel() * 4) / 2**20
    f_bwd = 2.5 * workloads.effective_flops(cfg, H)          # this rank's gradient products
    job = 2.5 * (workloads.effective_flops(cfg0) * (world if args.scaling == "weak" else 1))
    achieved = f_bwd / (step_ms * 1e-3) / 1e12
    value = job / (step_ms * 1e-3) / 1e12
    line = {
        "metric": "attention backward effective TFLOP/s (dQ, dK, dV; 10*S^2*D per head, causal halved), B200",
        "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world, "steps": n, "warmup": args.warmup,
        "ms_per_step": round(step_ms, 4), "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None,
        "dtype": "f16 (f32 accumulate)", "data": "synthetic",
        "config": {"workload": f"{args.config} shapes, unrouted: B{cfg0['B']} H{cfg0['H']} S{S} D{D}"
                               f"{' causal' if causal else ''}, backward from the training forward's LSE",
                   "B": cfg0["B"], "H": cfg0["H"], "S": S, "D": D, "causal": causal,
                   "parallelism": f"heads over {world} GPU rank(s) ({args.scaling}), no collective",
                   "l2": (f"inputs and outputs {footprint_mib:.0f} MiB per GPU, larger than L2 (126 MiB); no flush"
                          if footprint_mib > 126 else
                          f"inputs and outputs {footprint_mib:.0f} MiB per GPU fit in L2 (126 MiB): warm-L2 timing, "
                          f"no flush")},
        "per_gpu_heads": H,
        "training_forward_ms": round(fwd_ms, 4),
        "training_step_tflops": round(job * 3.5 / 2.5 / ((fwd_ms + step_ms) * 1e-3) / 1e12, 2),
        "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": peaks["bf16_tflops"],
                     "unit": "TFLOP/s", "frac": round(achieved / peaks["bf16_tflops"], 4),
                     "peak_source": f"{peaks['source']} bf16 dense (burst), MEASURED_PEAKS.json (fp16 runs at the "
                                    f"bf16 rate)",
                     "traffic": None,
                     "kernel": "backward_rows_kernel + backward_cols_kernel",
                     "work": "five gradient products (S recomputed counts once): 10*S^2*D per head, causal halved; "
                             "the kernels execute seven (S and dP in both kernels)"},
        "e2e": {"value": round(job * (3.5 / 2.5) / (e2e_ms * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
                "h2d_bytes_per_step": 4 * q.numel() * 2, "d2h_bytes_per_step": 3 * dq.numel() * 4,
                "ms_per_step": round(e2e_ms, 3),
                "api": "H2D of Q, K, V, dO; tilemix_attention_batched_lse; tilemix_attention_backward; D2H of dQ, "
                       "dK, dV (C-ABI, pinned host buffers); value counts forward + backward work"},
        "clocks": clk,
        "gpu_launches": 2 * n,
        "repo_native_so": repo_libraries(),
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    emit(line)


# ----------------------------------------------------------- reference arm
def run_reference(args, rank, world):
    """The reference's own CPU implementation of the path on the host cores,
    on this arm's config/metric; each step is a bounded sample."""
    if rank != 0:
        return
    import numpy as np
    import torch
    from tilemix_b200 import workloads
    cfg = workloads.config(args.config, p=args.p)
    # a few heads of the workload, drawn with the CPU generator (the sample uses whole heads)
    w = workloads.make_inputs(args.config, p=args.p, batch=1, heads=min(cfg["H"], 16))
    host = {"q": w["q"].numpy(), "k": w["k"].numpy(), "v": w["v"].numpy(), "words": w["words"].numpy()}
    values, walls = [], []
    last = None
    # Each step is one bounded sample of the workload (whole heads), so that
    # the whole run ends within a few minutes; the throughput of a sample is
    # the full workload's FLOPs over its extrapolated step time.
    per_step = max(0.5, min(args.cpu_seconds, 150.0 / (args.warmup + args.steps)))
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        last = cpu_reference_sample(host, cfg, per_step)
        wall = time.perf_counter() - t0
        if i >= args.warmup:
            values.append(last["step_seconds"])
            walls.append(wall)
    step_s = statistics.median(values)
    f_eff = workloads.effective_flops(cfg)
    value = f_eff / step_s / 1e12
    cpu = {"value": round(value, 6), "unit": "TFLOP/s", "cores": last["cores"], "kind": last["kind"],
           "sample": last["sample"]}
    line = {"metric": METRIC, "impl": "reference", "value": round(value, 6), "unit": "TFLOP/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            # time that actually ran per step: one bounded sample (steps x this is the timed wall time)
            "ms_per_step": round(statistics.median(walls) * 1e3, 1),
            "ms_per_step_basis": "wall time of one bounded sample step (whole heads), not of a full-workload step",
            "extrapolated_ms_per_full_step": round(step_s * 1e3, 1),
            "higher_is_better": True, "scaling": args.scaling,
            "vs_baseline": None, "dtype": "f64 (reference CPU emulation)", "data": "synthetic",
            "config": config_block(args, world),
            "cpu_baseline": cpu,
            "e2e": {"value": round(value, 6), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    gpu = reference_gpu_sample(args, cfg)
    if gpu is not None:
        line["reference_gpu"] = gpu
    line["repo_native_so"] = repo_libraries()
    emit(line)


def reference_gpu_sample(args, cfg, heads: int = 4, reps: int = 3):
    """The reference's own GPU kernels (src/tilemix.cu built for sm_100a, called
    per head through quantize_tilemix_qk + launch_fused_fp16_attention) on a few
    whole heads of the workload. The reference kernel has no causal mask, so the
    heads run non-causal and the value is 4*heads*S^2*D FLOP per second."""
    import torch
    import oracle
    from tilemix_b200 import workloads
    lib = oracle.ref_gpu_lib()
    if lib is None or not torch.cuda.is_available():
        return None
    w = workloads.make_inputs(args.config, p=args.p, batch=1, heads=heads, device="cuda")
    H, S, D = w["heads"], w["S"], w["D"]
    q, k, v = w["q"], w["k"], w["v"]
    words = w["words"].cuda()
    q8, k8 = torch.empty_like(q, dtype=torch.int8), torch.empty_like(k, dtype=torch.int8)
    qs = torch.empty((H, (S - 1) // 128 + 1), dtype=torch.float16, device="cuda")
    ks = torch.empty((H, (S - 1) // 64 + 1), dtype=torch.float16, device="cuda")
    out = torch.empty((H, S, D), dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream()

    def run():
        err = lib.ref_gpu_tilemix_heads(q.data_ptr(), k.data_ptr(), v.data_ptr(), q8.data_ptr(), k8.data_ptr(),
                                        qs.data_ptr(), ks.data_ptr(), out.data_ptr(), H, S, S, D,
                                        w["score_scale"], words.data_ptr(), words.numel() // H, 2,
                                        stream.cuda_stream)
        if err:
            raise SystemExit(f"reference GPU kernels returned cudaError {err}")

    run()
    torch.cuda.synchronize()
    times = []
    for _ in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        run()
        b.record(stream)
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b))
    ms = statistics.median(times)
    flops = 4.0 * H * S * S * D
    return {"value": round(flops / (ms * 1e-3) / 1e12, 4), "unit": "TFLOP/s", "ms_per_head": round(ms / H, 3),
            "sample": f"{H} whole heads of {args.config} shapes (S={S}, D={D}) through the reference's "
                      f"quantize_tilemix_qk + launch_fused_fp16_attention built for sm_100a, one call per "
                      f"head; non-causal (the reference kernel has no causal mask), median of {reps}"}


def main():
    args = parse_args()
    claim_stdout()
    rank, world, local = dist_setup(args)
    try:
        if args.op == "backward":
            if args.impl == "reference":
                if rank == 0:
                    emit({"impl": "reference", "unavailable": "the reference has no backward pass (forward only)"})
            else:
                run_backward(args, rank, world, local)
        elif args.impl == "reference":
            run_reference(args, rank, world)
        else:
            run_tilemix(args, rank, world, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
