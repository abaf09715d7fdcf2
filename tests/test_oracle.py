"""CPU: pin the C oracle against the reference's own CPU oracle.

Golden vectors in tests/golden/reference_golden.npz were produced by the
reference's src/tests/reference_tilemix.h / reference_attention.h (compiled in
place, see tests/golden/make_golden.py); when oracle/_ref is present the two
are also compared live on fresh random cases.
"""
import json
from pathlib import Path

import numpy as np
import pytest

import oracle
import refcases

GOLDEN = Path(__file__).resolve().parent / "golden" / "reference_golden.npz"


@pytest.fixture(scope="module")
def golden():
    g = np.load(GOLDEN)
    return g, json.loads(bytes(g["index"]).decode())


def test_half_conversion_matches_ieee():
    rng = np.random.default_rng(1)
    x = (rng.standard_normal(50000) * 10.0 ** rng.integers(-9, 6, 50000)).astype(np.float32)
    edge = np.array([65504, 65519.99, 65520, 65536, 1e-8, 2.0**-25, 2.0**-24, 3 * 2.0**-25,
                     2.0**-14, 2.0**-14 * 0.999, -0.0, 0.0, np.inf, -np.inf], np.float32)
    x = np.concatenate([x, edge])
    with np.errstate(over="ignore"):
        expect = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(oracle.float_to_half_bits(x), expect)
    lib = oracle.lib()
    for h in range(0, 65536, 7):
        if (h & 0x7C00) == 0x7C00 and (h & 0x3FF):
            continue   # NaN payloads
        assert lib.orc_half_to_float(h) == np.uint16(h).view(np.float16).astype(np.float32)


def test_rounding_ties_known_answer():
    """tilemix_test.cu:376,386-387: half AWAY from zero, not half-even."""
    q, _ = refcases.quant_inputs(129, 65, 1, "rounding")
    q8, _ = oracle.quantize(q, 128)
    assert q8.reshape(-1)[:8].tolist() == refcases.ROUNDING_KNOWN


def test_quantizer_vs_reference_golden(golden):
    g, index = golden
    for i, (m, n, d, pattern) in enumerate(index["quant"]):
        q, k = refcases.quant_inputs(m, n, d, pattern)
        q8, qs = oracle.quantize(q, 128)
        k8, ks = oracle.quantize(k, 64)
        assert np.array_equal(q8, g[f"quant{i}_q8"]), pattern
        assert np.array_equal(k8, g[f"quant{i}_k8"]), pattern
        assert np.array_equal(qs.view(np.uint16), g[f"quant{i}_qs"]), pattern
        assert np.array_equal(ks.view(np.uint16), g[f"quant{i}_ks"]), pattern


def test_dense_vs_reference_golden(golden):
    g, index = golden
    for i, (m, n, d, pattern, _) in enumerate(index["dense"]):
        q, k, v = refcases.inputs(m, n, d, pattern)
        out = oracle.dense_attention(q, k, v)
        np.testing.assert_allclose(out, g[f"dense{i}_o"], rtol=0, atol=1e-12, err_msg=pattern)


def test_routing_vs_reference_golden(golden):
    g, index = golden
    for i, (m, n, d, pattern, _, group, route, _) in enumerate(index["routing"]):
        q, k, v = refcases.inputs(m, n, d, pattern)
        q8, qs = oracle.quantize(q, 128)
        k8, ks = oracle.quantize(k, 64)
        words, bits = refcases.routing_words(m, n, group, "fp16" if route == "implicit-fp16" else route)
        assert np.array_equal(bits, g[f"routing{i}_bits"])
        assert np.array_equal(oracle.decode_routing(words, m, n, group), bits)
        scale = float(np.float32(1.0) / np.sqrt(np.float32(d)))
        out = oracle.tilemix_attention(q, k, v, q8, k8, qs, ks, bits, scale)
        np.testing.assert_allclose(out, g[f"routing{i}_o"], rtol=0, atol=1e-12,
                                   err_msg=f"{pattern} {route}")
        for (a, b), dot in zip(g[f"routing{i}_pairs"], g[f"routing{i}_dots"]):
            assert oracle.int8_dot(q8, k8, int(a), int(b)) == dot


def test_closed_form_patterns():
    """tilemix_test.cu:237-260 -- the dense oracle against closed-form softmax."""
    for pattern in ("rising", "falling", "alternating", "late-extreme", "negative"):
        n = 129 if pattern == "alternating" else 65
        q, k, v = refcases.inputs(17, n, 1, pattern)
        out = oracle.dense_attention(q, k, v)
        np.testing.assert_allclose(out, refcases.closed_form(pattern, v, n), rtol=1e-12, atol=1e-12)


def test_baseline_c1_vs_reference_golden(golden):
    g, _ = golden
    from tilemix_b200 import workloads
    w = workloads.make_inputs("c1")
    q, k, v = (w[x][0].numpy() for x in ("q", "k", "v"))
    q8, qs = oracle.quantize(q, 128)
    k8, ks = oracle.quantize(k, 64)
    assert np.array_equal(q8, g["c1_q8"]) and np.array_equal(k8, g["c1_k8"])
    assert np.array_equal(qs.view(np.uint16), g["c1_qs"]) and np.array_equal(ks.view(np.uint16), g["c1_ks"])
    assert np.array_equal(w["words"].numpy(), g["c1_words"])
    bits = oracle.decode_routing(g["c1_words"], 256, 256, 2)
    out = oracle.tilemix_attention(q, k, v, q8, k8, qs, ks, bits, w["score_scale"])
    np.testing.assert_allclose(out, g["c1_o"], rtol=0, atol=1e-12)


def test_routing_word_count_known_answers():
    """tilemix_test.cu:208-217."""
    rc = oracle.routing_word_count
    assert rc(17, 2048, 1) == 2 and rc(17, 2049, 1) == 4 and rc(17, 4097, 2) == 4
    assert rc(17, 4097, 1) == 6 and rc(17, 2**31 - 1, 2**31 - 1) == 2
    assert rc(0, 1, 1) == 0 and rc(1, 0, 1) == 0 and rc(1, 1, 0) == 0


@pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built (no reference tree)")
def test_oracle_vs_reference_live():
    rng = np.random.default_rng(11)
    for m, n, d in [(1, 1, 1), (129, 131, 17), (200, 77, 64), (33, 300, 128), (256, 256, 96)]:
        q = (rng.standard_normal((m, d)) * 2).astype(np.float16)
        k = (rng.standard_normal((n, d)) * 2).astype(np.float16)
        v = rng.standard_normal((n, d)).astype(np.float16)
        q8, qs = oracle.quantize(q, 128)
        k8, ks = oracle.quantize(k, 64)
        rq8, rqs = oracle.ref_quantize(q, 128)
        rk8, rks = oracle.ref_quantize(k, 64)
        assert np.array_equal(q8, rq8) and np.array_equal(k8, rk8)
        assert np.array_equal(qs.view(np.uint16), rqs.view(np.uint16))
        assert np.array_equal(ks.view(np.uint16), rks.view(np.uint16))
        routes = rng.integers(0, 2, ((m + 15) // 16, (n + 31) // 32)).astype(np.uint8)
        a = oracle.tilemix_attention(q, k, v, q8, k8, qs, ks, routes, 0.3)
        b = oracle.ref_tilemix(q, k, v, q8, qs, k8, ks, routes, 0.3)
        np.testing.assert_allclose(a, b, rtol=0, atol=1e-12)


@pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built (no reference tree)")
def test_causal_restatement_matches_reference_prefix_calls():
    """The causal extension equals the reference's own reference_tilemix run on
    each row's key prefix (how the CPU baseline drives the reference)."""
    rng = np.random.default_rng(5)
    h, m, d = 2, 300, 64
    q = rng.standard_normal((h, m, d)).astype(np.float16)
    k = rng.standard_normal((h, m, d)).astype(np.float16)
    v = rng.standard_normal((h, m, d)).astype(np.float16)
    q8, qs = oracle.quantize(q, 128)
    k8, ks = oracle.quantize(k, 64)
    routes = rng.integers(0, 2, (h, (m + 15) // 16, (m + 31) // 32)).astype(np.uint8)
    full = oracle.tilemix_attention(q, k, v, q8, k8, qs, ks, routes, 0.125, causal=True)
    rows = np.array([0, 1, 17, 128, 299])
    heads = np.array([1, 0])
    ref = oracle.tilemix_sampled(q, k, v, q8, k8, qs, ks, routes, heads, rows, 0.125, True,
                                 use_reference=True)
    np.testing.assert_allclose(ref, full[heads][:, rows], rtol=0, atol=1e-12)
