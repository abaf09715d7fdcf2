"""Generate tests/golden/reference_golden.npz from the reference's OWN CPU oracle.

Runs the reference's src/tests/reference_tilemix.h and reference_attention.h,
compiled in place into oracle/_ref/libtilemix_ref.so by oracle/build_ref.sh,
on the reference test suite's cases (tests/refcases.py) and stores:
  * quantizer cases: Q8/K8 bytes and fp16 scales (reference_quantize);
  * dense cases: fp64 outputs (reference_attention);
  * routing cases: fp64 mixed outputs (reference_tilemix) and sampled exact
    INT32 dots (reference_int8_dot);
  * BASELINE config 1 (B1 H1 S256 D64, seed 0, p=0.5): quantized operands and
    the fp64 mixed output.
The fixtures let machines without the reference tree pin the C oracle and the
CUDA path against the reference's own numbers.

Usage: python tests/golden/make_golden.py   (needs oracle/_ref built)
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parents[2]
for p in (REPO, REPO / "tests", REPO / "tilemix-cuda_b200"):
    sys.path.insert(0, str(p))

import oracle  # noqa: E402
import refcases  # noqa: E402

OUT = Path(__file__).resolve().parent / "reference_golden.npz"


def main() -> None:
    if not oracle.ref_available():
        oracle.build()
    assert oracle.ref_available(), "oracle/_ref/libtilemix_ref.so missing (reference tree needed)"
    arrays: dict[str, np.ndarray] = {}
    index: dict[str, list] = {"quant": [], "dense": [], "routing": []}

    for i, (m, n, d, pattern) in enumerate(refcases.QUANT_CASES):
        q, k = refcases.quant_inputs(m, n, d, pattern)
        q8, qs = oracle.ref_quantize(q, 128)
        k8, ks = oracle.ref_quantize(k, 64)
        arrays[f"quant{i}_q8"], arrays[f"quant{i}_qs"] = q8, qs.view(np.uint16)
        arrays[f"quant{i}_k8"], arrays[f"quant{i}_ks"] = k8, ks.view(np.uint16)
        index["quant"].append([m, n, d, pattern])

    for i, (m, n, d, pattern, default_stream) in enumerate(refcases.DENSE_CASES):
        q, k, v = refcases.inputs(m, n, d, pattern)
        arrays[f"dense{i}_o"] = oracle.ref_attention(q, k, v)
        index["dense"].append([m, n, d, pattern, default_stream])

    rng = np.random.default_rng(7)
    for i, ((m, n, d, pattern, default_stream), group, route, trace) in enumerate(refcases.routing_cases()):
        q, k, v = refcases.inputs(m, n, d, pattern)
        q8, qs = oracle.ref_quantize(q, 128)
        k8, ks = oracle.ref_quantize(k, 64)
        words, bits = refcases.routing_words(m, n, group, "fp16" if route == "implicit-fp16" else route)
        scale = np.float32(1.0) / np.sqrt(np.float32(d))
        arrays[f"routing{i}_o"] = oracle.ref_tilemix(q, k, v, q8, qs, k8, ks, bits, float(scale))
        pairs = np.stack([rng.integers(0, m, 16), rng.integers(0, n, 16)], axis=1)
        dots = np.array([oracle.ref_int8_dot(q8, k8, int(a), int(b)) for a, b in pairs], np.int32)
        arrays[f"routing{i}_pairs"], arrays[f"routing{i}_dots"] = pairs.astype(np.int32), dots
        arrays[f"routing{i}_bits"] = bits
        index["routing"].append([m, n, d, pattern, default_stream, group, route, trace])

    # BASELINE config 1 through the workload generator of the package.
    from tilemix_b200 import workloads
    w = workloads.make_inputs("c1")
    q, k, v = (w[x][0].numpy() for x in ("q", "k", "v"))
    q8, qs = oracle.ref_quantize(q, 128)
    k8, ks = oracle.ref_quantize(k, 64)
    bits = oracle.decode_routing(w["words"].numpy(), q.shape[0], k.shape[0], 2)
    arrays["c1_q8"], arrays["c1_qs"], arrays["c1_k8"], arrays["c1_ks"] = q8, qs.view(np.uint16), k8, ks.view(np.uint16)
    arrays["c1_words"] = w["words"].numpy()
    arrays["c1_o"] = oracle.ref_tilemix(q, k, v, q8, qs, k8, ks, bits, w["score_scale"])

    arrays["index"] = np.frombuffer(json.dumps(index).encode(), np.uint8)
    np.savez_compressed(OUT, **arrays)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
