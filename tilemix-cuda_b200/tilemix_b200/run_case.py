"""Run one BASELINE configuration (optionally shrunk) through the C-ABI: the
quantizer then the fused attention kernel, `--iters` times, and print the
per-kernel CUDA-event times. Used for ncu captures of a small case:

  python -m tilemix_b200.run_case --config c3 --batch 2 --iters 3
"""
from __future__ import annotations

import argparse
import json

import torch

import tilemix_b200 as tm
from tilemix_b200 import workloads


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--config", default="c3", choices=sorted(workloads.CONFIGS))
    ap.add_argument("--batch", type=int, default=None)
    ap.add_argument("--heads", type=int, default=None)
    ap.add_argument("--seq", type=int, default=None)
    ap.add_argument("--p", type=float, default=None)
    ap.add_argument("--iters", type=int, default=3)
    args = ap.parse_args()

    w = workloads.make_inputs(args.config, p=args.p, batch=args.batch, heads=args.heads,
                              seq=args.seq, device="cuda")
    H, S, D, cfg = w["heads"], w["S"], w["D"], w["cfg"]
    q, k, v = w["q"], w["k"], w["v"]
    words = w["words"].cuda()
    q8, k8, qs, ks = tm.quantize(q, k)
    out = torch.empty((H, S, D), dtype=torch.float32, device="cuda")
    routing = tm.TileMixRouting(words, words.numel(), 2)
    quantized = tm.TileMixQuantized(q8, k8, qs, ks)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3 * args.iters)]
    for i in range(args.iters):
        ev[3 * i].record()
        tm.check(tm.quantize_tilemix_qk_batched(q, k, q8, k8, qs, ks, H, S, S, D), "quantize")
        ev[3 * i + 1].record()
        tm.check(tm.tilemix_attention_batched(q, k, v, out, H, S, S, D, w["score_scale"],
                                              cfg["causal"], None, routing, quantized), "attention")
        ev[3 * i + 2].record()
    torch.cuda.synchronize()
    err, status = tm.read_and_clear_status()
    tm.check(err, "status read")
    if status:
        raise SystemExit(f"kernel watchdog status {status:#x}")
    f_eff = workloads.effective_flops(cfg, H)
    quant_ms = [ev[3 * i].elapsed_time(ev[3 * i + 1]) for i in range(args.iters)]
    attn_ms = [ev[3 * i + 1].elapsed_time(ev[3 * i + 2]) for i in range(args.iters)]
    print(json.dumps({"config": args.config, "heads": H, "S": S, "D": D,
                      "quantize_ms": quant_ms, "attention_ms": attn_ms,
                      "attention_tflops": [f_eff / (t * 1e-3) / 1e12 for t in attn_ms]}))


if __name__ == "__main__":
    main()
