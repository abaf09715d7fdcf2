"""The dense cross-check against the reference's own Python oracle
(python/reference_attention.py:11-25): fixtures it generated
(tests/golden/make_dense_golden.py) for seeded fp16 inputs of small and ragged
shapes and its self-check patterns (uniform, extreme logits).

CPU: the C oracle's dense attention equals the reference Python in fp64.
GPU: the fused kernel with every tile FP16 (no routing) matches it within the
reference suite's own tolerance (atol 1e-5, rtol 1e-4) and the north-star bar.
"""
from pathlib import Path

import numpy as np
import pytest

import oracle

GOLDEN = Path(__file__).resolve().parent / "golden" / "reference_python_dense.npz"


def _cases():
    g = np.load(GOLDEN)
    for name in g["names"]:
        yield str(name), g[f"{name}_q"], g[f"{name}_k"], g[f"{name}_v"], g[f"{name}_o64"], g[f"{name}_o32"]


def test_oracle_dense_attention_equals_reference_python():
    for name, q, k, v, o64, o32 in _cases():
        got = oracle.dense_attention(q, k, v)
        assert np.abs(got - o64).max() <= 1e-12 * max(1.0, np.abs(o64).max()), name
        assert np.abs(o32.astype(np.float64) - o64).max() <= 1e-4, name   # the reference's fp32 mode agrees too


@pytest.mark.gpu
def test_fused_kernel_all_fp16_matches_reference_python():
    import torch
    import tilemix_b200 as tm
    for name, q, k, v, o64, _ in _cases():
        out = tm.attention(*(torch.from_numpy(x).cuda() for x in (q, k, v)), score_scale=1.0 / np.sqrt(q.shape[1]))
        torch.cuda.synchronize()
        got = out.cpu().numpy().astype(np.float64)
        diff = np.abs(got - o64)
        assert (diff <= 1e-5 + 1e-4 * np.abs(o64)).all(), (name, float(diff.max()))
        assert diff.max() <= 2e-3 and np.linalg.norm(diff) <= 1e-3 * max(np.linalg.norm(o64), 1e-30), name
    err, status = tm.read_and_clear_status()
    assert err == 0 and status == 0
