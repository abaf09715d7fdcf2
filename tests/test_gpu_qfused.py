"""GPU: Q quantization fused into the attention kernel (tilemix_attention_batched_qfused).

Parity is bit-exact and chained to the oracle:
  * the Q8 bytes and fp16 scales the kernel writes equal the oracle's
    restatement of the reference quantizer (and the standalone quantizer's);
  * the K-only quantizer equals the K half of the oracle's quantization;
  * the output equals, bit for bit, tilemix_attention_batched fed the
    standalone quantizer's operands, whose own parity with the oracle the other
    attention tests check (and this file checks against the oracle too).
Cases: the reference's routing shapes and head-dim sweep (TMA and plain-load
paths, ragged M and N, every key_tiles_per_group), the quantizer's special
patterns (ties, tiny, max-range, block outliers) and batched causal configs.
"""
import math

import numpy as np
import pytest
import torch

import oracle
import refcases
from gpu_util import I8_GUARD, SCALE_GUARD, dev, guarded, host
import tilemix_b200 as tm
from tilemix_b200 import workloads

pytestmark = pytest.mark.gpu


def run_both(q, k, v, words, m, n, d, group, scale, causal, heads):
    """(fused O, fused Q8 with guards, fused q scales with guards, K8, k scales,
    regular O, regular Q8, regular q scales)."""
    qd, kd, vd = dev(q), dev(k), dev(v)
    wd = dev(words)
    qb, kb = (m - 1) // 128 + 1, (n - 1) // 64 + 1
    # regular path
    rq8 = torch.empty(q.size, dtype=torch.int8, device="cuda")
    rk8 = torch.empty(k.size, dtype=torch.int8, device="cuda")
    rqs = torch.empty(heads * qb, dtype=torch.float16, device="cuda")
    rks = torch.empty(heads * kb, dtype=torch.float16, device="cuda")
    ro = torch.empty(q.size, dtype=torch.float32, device="cuda")
    assert tm.quantize_tilemix_qk_batched(qd, kd, rq8, rk8, rqs, rks, heads, m, n, d) == 0
    routing = tm.TileMixRouting(wd, wd.numel(), group)
    assert tm.tilemix_attention_batched(qd, kd, vd, ro, heads, m, n, d, scale, causal, None, routing,
                                        tm.TileMixQuantized(rq8, rk8, rqs, rks)) == 0
    # fused path, outputs guarded
    k8 = guarded(k.size, torch.int8, I8_GUARD)
    ks = guarded(heads * kb, torch.float16, SCALE_GUARD)
    q8 = guarded(q.size, torch.int8, I8_GUARD)
    qs = guarded(heads * qb, torch.float16, SCALE_GUARD)
    o = torch.full((q.size,), float("nan"), dtype=torch.float32, device="cuda")
    assert tm.quantize_tilemix_k_batched(kd, k8[1:], ks[1:], heads, n, d) == 0
    assert tm.tilemix_attention_batched_qfused(qd, kd, vd, o, heads, m, n, d, scale, causal, None, routing,
                                               k8[1:], ks[1:], q8[1:], qs[1:]) == 0
    # and without the optional outputs
    o2 = torch.full((q.size,), float("nan"), dtype=torch.float32, device="cuda")
    assert tm.tilemix_attention_batched_qfused(qd, kd, vd, o2, heads, m, n, d, scale, causal, None, routing,
                                               k8[1:], ks[1:]) == 0
    torch.cuda.synchronize()
    assert torch.equal(o.view(torch.int32), o2.view(torch.int32))
    assert np.array_equal(host(qd).view(np.uint16), q.view(np.uint16)), "inputs modified"
    assert np.array_equal(host(kd).view(np.uint16), k.view(np.uint16)), "inputs modified"
    return tuple(host(t) for t in (o, q8, qs, k8, ks, ro, rq8, rqs))


def check(q, k, v, words, m, n, d, group, scale, causal=False, heads=1):
    o, q8, qs, k8, ks, ro, rq8, rqs = run_both(q, k, v, words, m, n, d, group, scale, causal, heads)
    for a, gv in ((q8, I8_GUARD), (k8, I8_GUARD), (qs, SCALE_GUARD), (ks, SCALE_GUARD)):
        assert a[0] == gv and a[-1] == gv, "guard overwritten"
    q3 = q.reshape(heads, m, d)
    k3 = k.reshape(heads, n, d)
    eq8, eqs = zip(*(oracle.quantize(q3[h], 128) for h in range(heads)))
    ek8, eks = zip(*(oracle.quantize(k3[h], 64) for h in range(heads)))
    assert np.array_equal(q8[1:-1], np.concatenate([a.reshape(-1) for a in eq8]))
    assert np.array_equal(qs[1:-1].view(np.uint16), np.concatenate([a.reshape(-1) for a in eqs]).view(np.uint16))
    assert np.array_equal(k8[1:-1], np.concatenate([a.reshape(-1) for a in ek8]))
    assert np.array_equal(ks[1:-1].view(np.uint16), np.concatenate([a.reshape(-1) for a in eks]).view(np.uint16))
    assert np.array_equal(q8[1:-1], rq8) and np.array_equal(qs[1:-1].view(np.uint16), rqs.view(np.uint16))
    assert np.array_equal(o.view(np.uint32), ro.view(np.uint32)), "fused output differs from the regular path"
    return o


@pytest.mark.parametrize("case", range(len(refcases.ROUTING_SHAPES) * 2))
def test_reference_routing_shapes(case):
    (m, n, d, pattern, _), group = refcases.ROUTING_SHAPES[case // 2]
    rp = ("mixed", "int8-requested")[case % 2]
    q, k, v = refcases.inputs(m, n, d, pattern)
    words, bits = refcases.routing_words(m, n, group, rp)
    scale = 1.0 / math.sqrt(d)
    o = check(q, k, v, words, m, n, d, group, scale)
    eq8, eqs = oracle.quantize(q, 128)
    ek8, eks = oracle.quantize(k, 64)
    expect = oracle.tilemix_attention(q, k, v, eq8, ek8, eqs, eks, bits, scale)
    diff = np.abs(o.astype(np.float64).reshape(m, d) - expect)
    assert diff.max() <= refcases.MAX_ABS_TOL


@pytest.mark.parametrize("d", refcases.ROUTING_D_SWEEP + [80, 96])
def test_head_dim_sweep(d):
    m, n = 300, 161
    rng = np.random.default_rng(d)
    q, k, v = (rng.standard_normal((x, d)).astype(np.float16) for x in (m, n, n))
    words, _ = refcases.routing_words(m, n, 1, "mixed")
    check(q, k, v, words, m, n, d, 1, 1.0 / math.sqrt(d))


@pytest.mark.parametrize("pattern", ["zeros", "rounding", "tiny", "max-range", "block-outliers"])
def test_quantizer_patterns(pattern):
    m, n, d = 257, 130, 64
    q, k = refcases.quant_inputs(m, n, d, pattern)
    v = np.random.default_rng(1).standard_normal((n, d)).astype(np.float16)
    words, _ = refcases.routing_words(m, n, 2, "int8-requested")
    check(q, k, v, words, m, n, d, 2, 0.0 if pattern == "max-range" else 0.125)


@pytest.mark.parametrize("name,heads,seq", [("c3", 4, 640), ("c5", 3, 512), ("c2", 2, 384)])
def test_batched_configs(name, heads, seq):
    w = workloads.make_inputs(name, batch=1, heads=heads, seq=seq)
    cfg = w["cfg"]
    q, k, v = (w[x].numpy() for x in ("q", "k", "v"))
    check(q, k, v, w["words"].numpy(), seq, seq, w["D"], 2, w["score_scale"], cfg["causal"], heads)


def test_argument_contract():
    q = torch.zeros((2, 128, 64), dtype=torch.float16, device="cuda")
    k8 = torch.zeros((2, 128, 64), dtype=torch.int8, device="cuda")
    ks = torch.zeros((2, 2), dtype=torch.float16, device="cuda")
    o = torch.empty((2, 128, 64), dtype=torch.float32, device="cuda")
    words = torch.zeros(2 * tm.tilemix_routing_word_count(128, 128, 2), dtype=torch.int64, device="cuda")
    r = tm.TileMixRouting(words, words.numel(), 2)
    f = tm.tilemix_attention_batched_qfused
    assert f(q, q, q, o, 2, 128, 128, 64, 0.1, False, None, r, k8, ks) == 0
    assert f(q, q, q, o, 2, 128, 128, 64, 0.1, False, None, tm.TileMixRouting(None, 0, 2), k8, ks) == 1
    assert f(q, q, q, o, 2, 128, 128, 64, 0.1, False, None, r, None, ks) == 1
    assert f(q, q, q, o, 2, 128, 128, 64, 0.1, False, None, r, k8, None) == 1
    assert f(q, q, q, o, 2, 128, 128, 64, float("nan"), False, None, r, k8, ks) == 1
    assert f(q, q, q, o, 2, 128, 128, 129, 0.1, False, None, r, k8, ks) == 801
    short = tm.TileMixRouting(words, words.numel() - 1, 2)
    assert f(q, q, q, o, 2, 128, 128, 64, 0.1, False, None, short, k8, ks) == 1
    torch.cuda.synchronize()
    err, status = tm.read_and_clear_status()
    assert err == 0 and status == 0


def test_nan_and_inf_tiles_match_the_standalone_quantizer():
    """Query tiles holding a NaN or an inf take the exact element-wise path in
    the fused quantization, as in the standalone quantizer: same Q8 bytes,
    same scales, and the same output bits as the unfused path."""
    m, n, d = 384, 200, 128
    rng = np.random.default_rng(4)
    q, k, v = (rng.standard_normal((x, d)).astype(np.float16) for x in (m, n, n))
    q[3, 9] = np.nan          # tile 0
    q[200, 0] = np.inf        # tile 1
    words, _ = refcases.routing_words(m, n, 2, "int8-requested")
    o, q8, qs, k8, ks, ro, rq8, rqs = run_both(q, k, v, words, m, n, d, 2, 0.09, False, 1)
    assert np.array_equal(q8[1:-1], rq8) and np.array_equal(qs[1:-1].view(np.uint16), rqs.view(np.uint16))
    assert np.isinf(qs[2]) and not q8[1:-1].reshape(m, d)[128:256].any()
    assert np.array_equal(o.view(np.uint32), ro.view(np.uint32))
