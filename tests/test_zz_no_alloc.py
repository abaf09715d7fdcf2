"""tilemix_attention_routed_noalloc: routed attention that allocates nothing.

Some callers cannot allocate device memory (an operator or plugin interface
handed only its inputs and outputs at launch time, a binding with no access to
the process's device allocator, a framework whose allocator owns the device).
This entry point keeps the INT8 copies of Q and K and their scales in a fixed
array of device memory inside the library. Its output must match the regular
path (quantize_tilemix_qk_batched into caller buffers, then
tilemix_attention_batched) within the parity tolerance, on calls in a row that
reuse the shared array with different shapes.

This file is collected last (its name sorts after the other test files).
"""
import math

import numpy as np
import pytest
import torch

import tilemix_b200 as tm
from tilemix_b200 import workloads

MAX_ABS, REL_L2 = 2e-3, 1e-3      # the parity tolerance of every output test


def test_oversized_problem_is_rejected_before_any_device_work():
    """INT8 copies beyond the scratch size return cudaErrorMemoryAllocation;
    the size check comes before any CUDA call, so this runs without a GPU."""
    heads, s, d = 129, 4096, 128          # 2 * 129 * 4096 * 128 bytes > 64 MiB
    assert 2 * heads * s * d > tm.NOALLOC_SCRATCH_BYTES
    wc = heads * tm.tilemix_routing_word_count(s, s, 2)
    fake = 1 << 20                       # never dereferenced: the call returns first
    routing = tm.TileMixRouting(fake, wc, 2)
    err = tm.tilemix_attention_routed_noalloc(fake, fake, fake, fake, heads, s, s, d, 0.088, True, routing)
    assert err == tm.cudaErrorMemoryAllocation


def _regular_path(w, causal):
    q, k, v = (w[n].cuda() for n in ("q", "k", "v"))
    words = w["words"].cuda()
    H, S, D = w["heads"], w["S"], w["D"]
    q8, k8 = torch.empty_like(q, dtype=torch.int8), torch.empty_like(k, dtype=torch.int8)
    qs = torch.empty((H, (S - 1) // 128 + 1), dtype=torch.float16, device="cuda")
    ks = torch.empty((H, (S - 1) // 64 + 1), dtype=torch.float16, device="cuda")
    out = torch.empty((H, S, D), dtype=torch.float32, device="cuda")
    tm.check(tm.quantize_tilemix_qk_batched(q, k, q8, k8, qs, ks, H, S, S, D), "quantize")
    tm.check(tm.tilemix_attention_batched(q, k, v, out, H, S, S, D, w["score_scale"], causal, None,
                                          tm.TileMixRouting(words, words.numel(), 2),
                                          tm.TileMixQuantized(q8, k8, qs, ks)), "attention")
    return q, k, v, words, out


@pytest.mark.gpu
def test_noalloc_matches_the_regular_entry_point_on_calls_in_a_row():
    cases = [  # (config, heads, seq, causal): different sizes, so the second call reuses the array differently
        ("c3", 4, 512, True),
        ("c2", 3, 320, False),
    ]
    for name, heads, seq, causal in cases:
        w = workloads.make_inputs(name, batch=1, heads=heads, seq=seq)
        q, k, v, words, expect = _regular_path(w, causal)
        got = torch.full_like(expect, float("nan"))
        H, S, D = w["heads"], w["S"], w["D"]
        err = tm.tilemix_attention_routed_noalloc(q, k, v, got, H, S, S, D, w["score_scale"], causal,
                                                  tm.TileMixRouting(words, words.numel(), 2))
        assert err == 0, err
        torch.cuda.synchronize()
        e, g = expect.cpu().double().numpy(), got.cpu().double().numpy()
        assert np.isfinite(g).all(), name
        diff = np.abs(g - e)
        rel = float(np.linalg.norm(diff) / np.linalg.norm(e))
        assert diff.max() <= MAX_ABS and rel <= REL_L2, (name, float(diff.max()), rel)
    err, status = tm.read_and_clear_status()
    assert err == 0 and status == 0, (err, status)
