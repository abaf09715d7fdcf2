"""GPU parity of the fused attention kernel through the C-ABI.

Mirrors the reference suite (src/tests/tilemix_test.cu): dense cases vs the
reference's fp64 outputs (golden), analytic score-scale/reuse checks, and the
routing cases with exact INT32 dots, exact decoded routing bits, guard
sentinels, input immutability, all-FP16 == unrouted bit-for-bit, and the
mixed output vs the reference's mixed-precision emulation. Tolerance (fp16 P
in a tensor-core PV MMA): max-abs 2e-3 and relative-L2 1e-3, refcases.MAX_ABS_TOL /
REL_L2_TOL.
"""
import json
import math
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
import refcases
from refcases import MAX_ABS_TOL, REL_L2_TOL, compare_stats
from gpu_util import (DEV, BITS_GUARD, DOT_GUARD, OUT_GUARD, dev, guarded, host, quantize_gpu)
import tilemix_b200 as tm

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden" / "reference_golden.npz"


@pytest.fixture(scope="module")
def golden():
    g = np.load(GOLDEN)
    return g, json.loads(bytes(g["index"]).decode())


def assert_close(actual, expected, what=""):
    max_abs, rel_l2 = compare_stats(actual, expected)
    assert np.isfinite(actual).all(), f"{what}: non-finite output"
    assert max_abs <= MAX_ABS_TOL and rel_l2 <= REL_L2_TOL, f"{what}: max_abs={max_abs:.3g} rel_l2={rel_l2:.3g}"


def run_dense(q, k, v, scale, stream=None):
    m, d = q.shape
    n = k.shape[0]
    qd, kd, vd = dev(q), dev(k), dev(v)
    out = guarded(m * d, torch.float32, OUT_GUARD, fill=float("nan"))
    assert tm.launch_fused_fp16_attention(qd, kd, vd, out[1:], m, n, d, scale, stream) == 0
    torch.cuda.synchronize()
    o = host(out)
    assert o[0] == OUT_GUARD and o[-1] == OUT_GUARD, "output guard overwritten"
    for t, a in ((qd, q), (kd, k), (vd, v)):
        assert np.array_equal(host(t), a), "kernel modified an input"
    return o[1:-1].reshape(m, d)


def test_dense_reference_cases(golden):
    g, index = golden
    stream = torch.cuda.Stream()
    for i, (m, n, d, pattern, default_stream) in enumerate(index["dense"]):
        q, k, v = refcases.inputs(m, n, d, pattern)
        scale = float(np.float32(1.0) / np.sqrt(np.float32(d)))
        out = run_dense(q, k, v, scale, None if default_stream else stream)
        assert_close(out, g[f"dense{i}_o"], f"M={m} N={n} d={d} {pattern}")


def test_score_scale_sweep_and_buffer_reuse():
    """tilemix_test.cu:330-355: closed form (2a + 4 + 8b)/(a + 1 + b), a=e^-s, b=e^s."""
    q = np.array([[1.0]], np.float16)
    k = np.array([[-1.0], [0.0], [1.0]], np.float16)
    v = np.array([[2.0], [4.0], [8.0]], np.float16)
    qd, kd, vd = dev(q), dev(k), dev(v)
    out = guarded(1, torch.float32, OUT_GUARD, fill=float("nan"))
    stream = torch.cuda.Stream()
    for s in (1.0, 0.0, -1.0, 0.5):
        assert tm.launch_fused_fp16_attention(qd, kd, vd, out[1:], 1, 3, 1, s, stream) == 0
        stream.synchronize()
        o = host(out)
        assert o[0] == OUT_GUARD and o[2] == OUT_GUARD
        a, b = math.exp(-s), math.exp(s)
        assert abs(o[1] - (2 * a + 4 + 8 * b) / (a + 1 + b)) <= MAX_ABS_TOL


def routing_case(g, i, shape, group, route, trace):
    m, n, d, pattern, default_stream = shape
    q, k, v = refcases.inputs(m, n, d, pattern)
    implicit = route == "implicit-fp16"
    words, bits = refcases.routing_words(m, n, group, "fp16" if implicit else route)
    stream = None if default_stream else torch.cuda.Stream()
    q8, k8, qs, ks = quantize_gpu(q, k, stream=stream)
    eq8, eqs = oracle.quantize(q, 128)
    ek8, eks = oracle.quantize(k, 64)
    assert np.array_equal(q8, eq8) and np.array_equal(k8, ek8)
    assert np.array_equal(qs.view(np.uint16), eqs.view(np.uint16))
    assert np.array_equal(ks.view(np.uint16), eks.view(np.uint16))
    qd, kd, vd = dev(q), dev(k), dev(v)
    q8d, k8d, qsd, ksd = dev(q8), dev(k8), dev(qs), dev(ks)
    wd = dev(words)
    scale = float(np.float32(1.0) / np.sqrt(np.float32(d)))
    out = guarded(m * d, torch.float32, OUT_GUARD, fill=float("nan"))
    # unrouted baseline on the same buffer
    assert tm.launch_fused_fp16_attention(qd, kd, vd, out[1:], m, n, d, scale, stream) == 0
    torch.cuda.synchronize()
    baseline = host(out).copy()
    bits_buf = guarded(bits.size, torch.uint8, BITS_GUARD)
    dots = guarded(m * n, torch.int32, DOT_GUARD)
    routing = tm.TileMixRouting(None if implicit else wd, 0 if implicit else words.size, group,
                                bits_buf[1:] if trace else None)
    quantized = tm.TileMixQuantized(q8d, k8d, qsd, ksd, dots[1:])
    assert tm.launch_fused_fp16_attention(qd, kd, vd, out[1:], m, n, d, scale, stream,
                                          routing, quantized) == 0
    torch.cuda.synchronize()
    o = host(out)
    assert o[0] == OUT_GUARD and o[-1] == OUT_GUARD, "routed output guard overwritten"
    what = f"M={m} N={n} d={d} {pattern} g={group} {route}"
    if not bits.any():
        assert np.array_equal(o.view(np.uint32), baseline.view(np.uint32)), f"{what}: all-FP16 != unrouted"
    dh = host(dots)
    assert dh[0] == DOT_GUARD and dh[-1] == DOT_GUARD
    int8_mask = np.repeat(np.repeat(bits, 16, axis=0)[:m], 32, axis=1)[:, :n].astype(bool)
    expect_dots = np.where(int8_mask, oracle.int8_dots(q8, k8), DOT_GUARD)
    assert np.array_equal(dh[1:-1].reshape(m, n), expect_dots), f"{what}: INT32 dots"
    bh = host(bits_buf)
    assert bh[0] == BITS_GUARD and bh[-1] == BITS_GUARD
    assert np.array_equal(bh[1:-1].reshape(bits.shape), bits if trace else np.full_like(bits, BITS_GUARD)), \
        f"{what}: decoded bits"
    assert np.array_equal(host(wd), words), "routing mask modified"
    for t, a in ((q8d, q8), (k8d, k8), (qsd, qs), (ksd, ks), (qd, q), (kd, k), (vd, v)):
        assert np.array_equal(host(t), a), f"{what}: operand modified"
    assert_close(o[1:-1].reshape(m, d), g[f"routing{i}_o"], what)


def test_routing_reference_cases(golden):
    g, index = golden
    for i, (m, n, d, pattern, default_stream, group, route, trace) in enumerate(index["routing"]):
        routing_case(g, i, (m, n, d, pattern, default_stream), group, route, trace)


def batched_case(heads, m, n, d, causal, p, seed, scale=None, tol_only=False):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((heads, m, d)).astype(np.float16)
    k = rng.standard_normal((heads, n, d)).astype(np.float16)
    v = rng.standard_normal((heads, n, d)).astype(np.float16)
    qd, kd, vd = dev(q), dev(k), dev(v)
    q8d, k8d, qsd, ksd = tm.quantize(qd, kd)
    qt, kt = (m + 15) // 16, (n + 31) // 32
    routes = (rng.random((heads, qt, (kt + 1) // 2)) < p).astype(np.uint8)
    words = np.concatenate([_pack(routes[h], m, n) for h in range(heads)])
    bits = np.stack([oracle.decode_routing(words[h * (words.size // heads):(h + 1) * (words.size // heads)],
                                           m, n, 2) for h in range(heads)])
    scale = scale if scale is not None else 1.0 / math.sqrt(d)
    out = tm.attention(qd, kd, vd, q8=q8d, k8=k8d, q_scales=qsd, k_scales=ksd, words=dev(words),
                       key_tiles_per_group=2, score_scale=scale, causal=causal)
    torch.cuda.synchronize()
    expect = oracle.tilemix_attention(q, k, v, host(q8d), host(k8d), host(qsd), host(ksd), bits,
                                      scale, causal)
    assert_close(host(out), expect, f"heads={heads} M={m} N={n} d={d} causal={causal} p={p}")


def _pack(group_bits, m, n):
    """Per-query-tile group bits [qt, groups] -> words with g=2."""
    qt, groups = group_bits.shape
    wpr = (groups + 63) // 64
    words = np.zeros(qt * wpr, np.uint64)
    for t in range(qt):
        for gi in range(groups):
            if group_bits[t, gi]:
                words[t * wpr + gi // 64] |= np.uint64(1) << np.uint64(gi % 64)
    return words


@pytest.mark.parametrize("heads,m,n,d,causal,p", [
    (3, 300, 300, 64, False, 0.5), (3, 300, 300, 64, True, 0.5), (2, 512, 512, 128, True, 0.75),
    (2, 640, 384, 128, False, 0.3), (1, 1000, 1000, 96, True, 1.0), (2, 129, 700, 48, False, 0.0),
    (4, 256, 256, 128, False, 0.5), (1, 2048, 2048, 128, True, 0.5),
])
def test_batched_and_causal(heads, m, n, d, causal, p):
    batched_case(heads, m, n, d, causal, p, seed=heads * 1000 + m + d)


def test_baseline_c1_full(golden):
    g, _ = golden
    from tilemix_b200 import workloads
    w = workloads.make_inputs("c1")
    q, k, v = (w[x][0].numpy() for x in ("q", "k", "v"))
    q8, k8, qs, ks = quantize_gpu(q, k)
    assert np.array_equal(q8, g["c1_q8"]) and np.array_equal(k8, g["c1_k8"])
    assert np.array_equal(qs.view(np.uint16), g["c1_qs"]) and np.array_equal(ks.view(np.uint16), g["c1_ks"])
    out = guarded(q.size, torch.float32, OUT_GUARD)
    routing = tm.TileMixRouting(dev(g["c1_words"]), g["c1_words"].size, 2)
    quantized = tm.TileMixQuantized(dev(q8), dev(k8), dev(qs), dev(ks))
    assert tm.launch_fused_fp16_attention(dev(q), dev(k), dev(v), out[1:], 256, 256, 64, w["score_scale"],
                                          None, routing, quantized) == 0
    torch.cuda.synchronize()
    o = host(out)
    assert o[0] == OUT_GUARD and o[-1] == OUT_GUARD
    assert_close(o[1:-1].reshape(256, 64), g["c1_o"], "BASELINE c1")
