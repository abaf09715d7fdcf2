"""Generates tests/golden/reference_python_dense.npz from the reference's own
Python oracle, python/reference_attention.py (reference_attention, fp64 and
fp32 compute), imported where it lies. Run on a machine holding the reference
tree (TILEMIX_REFERENCE_ROOT, else the reference_path of BASELINE.json); the
fixtures are committed so the tests need no reference tree.

The reference's Python file is its dense cross-check (all tiles FP16 must
match dense attention); the inputs are seeded fp16 N(0,1) draws of small and
ragged shapes, plus its uniform / single-key / extreme-logit patterns.
"""
from __future__ import annotations

import importlib.util
import json
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
SHAPES = [(1, 1, 1), (3, 5, 7), (17, 33, 17), (64, 64, 32), (130, 257, 128), (300, 1000, 64), (129, 4097, 16)]


def reference_module():
    root = os.environ.get("TILEMIX_REFERENCE_ROOT") or json.loads((REPO / "BASELINE.json").read_text())["reference_path"]
    path = Path(root) / "python" / "reference_attention.py"
    spec = importlib.util.spec_from_file_location("reference_attention", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main() -> None:
    ref = reference_module()
    g = torch.Generator(device="cpu").manual_seed(20261202)
    out = {}
    cases = []
    for i, (m, n, d) in enumerate(SHAPES):
        q, k, v = (torch.randn((x, d), generator=g).half() for x in (m, n, n))
        cases.append((f"rand{i}", q, k, v))
    # the patterns of the reference's self_check (python/reference_attention.py:40-47)
    cases.append(("uniform", torch.zeros((3, 7), dtype=torch.float16), torch.ones((5, 7), dtype=torch.float16),
                  torch.arange(35, dtype=torch.float16).reshape(5, 7)))
    cases.append(("extreme", torch.tensor([[1000.0]], dtype=torch.float16),
                  torch.tensor([[1000.0], [-1000.0]], dtype=torch.float16), torch.tensor([[3.0], [-7.0]], dtype=torch.float16)))
    names = []
    for name, q, k, v in cases:
        names.append(name)
        out[f"{name}_q"], out[f"{name}_k"], out[f"{name}_v"] = (t.numpy() for t in (q, k, v))
        out[f"{name}_o64"] = ref.reference_attention(q, k, v, compute_dtype=torch.float64).numpy()
        out[f"{name}_o32"] = ref.reference_attention(q, k, v, compute_dtype=torch.float32).numpy()
    out["names"] = np.array(names)
    np.savez_compressed(HERE / "reference_python_dense.npz", **out)
    print(f"wrote {len(names)} cases to {HERE / 'reference_python_dense.npz'}")


if __name__ == "__main__":
    sys.exit(main())
