"""GPU parity at the BASELINE configurations' full sizes.

C1 and C2 are checked in full against the fp64 oracle. C3 (B8 H32 S4096 D128,
causal, outliers), C4 (S=32768 at INT8 fractions 0, 0.5, 1) and C5 (INT8
fraction sweep with a forced-FP16 diagonal band) run in full on the GPU;
the quantized tensors are compared bit-for-bit in full, the outputs on a
fixed sample of (head, row) pairs (rows are independent), plus
size-independent properties: an all-FP16 mask reproduces the unrouted output
bit-for-bit, and a constant V gives a constant output (softmax rows sum to 1).
Inputs come from the seeded CPU generator in tilemix_b200.workloads.
"""
import numpy as np
import pytest
import torch

import oracle
from refcases import MAX_ABS_TOL, REL_L2_TOL, compare_stats
import tilemix_b200 as tm
from tilemix_b200 import workloads

pytestmark = pytest.mark.gpu


def run_config(w, words=None):
    H, S, D, cfg = w["heads"], w["S"], w["D"], w["cfg"]
    q, k, v = (w[x].cuda() for x in ("q", "k", "v"))
    q8, k8, qs, ks = tm.quantize(q, k)
    wd = (w["words"] if words is None else words).cuda()
    out = tm.attention(q, k, v, q8=q8, k8=k8, q_scales=qs, k_scales=ks, words=wd, key_tiles_per_group=2,
                       score_scale=w["score_scale"], causal=cfg["causal"])
    torch.cuda.synchronize()
    err, status = tm.read_and_clear_status()
    assert err == 0 and status == 0
    return out, (q8, k8, qs, ks), (q, k, v)


def check_quantized(w, quant):
    q8, k8, qs, ks = (t.cpu().numpy() for t in quant)
    eq8, eqs = oracle.quantize(w["q"].numpy(), 128)
    ek8, eks = oracle.quantize(w["k"].numpy(), 64)
    assert np.array_equal(q8, eq8) and np.array_equal(k8, ek8)
    assert np.array_equal(qs.view(np.uint16), eqs.view(np.uint16))
    assert np.array_equal(ks.view(np.uint16), eks.view(np.uint16))
    return q8, k8, qs, ks


def sampled_check(w, out, quant_host, heads, rows):
    H, S = w["heads"], w["S"]
    q8, k8, qs, ks = quant_host
    wc = w["words"].numel() // H
    words = w["words"].numpy()
    bits = np.stack([oracle.decode_routing(words[h * wc:(h + 1) * wc], S, S, 2) for h in heads])
    sel = lambda t: np.ascontiguousarray(t.numpy()[heads])
    expect = oracle.tilemix_sampled(sel(w["q"]), sel(w["k"]), sel(w["v"]), q8[heads], k8[heads],
                                    qs[heads], ks[heads], bits, np.arange(len(heads)), rows,
                                    w["score_scale"], w["cfg"]["causal"])
    actual = out.cpu().numpy()[heads][:, rows]
    max_abs, rel_l2 = compare_stats(actual, expect)
    assert np.isfinite(actual).all()
    assert max_abs <= MAX_ABS_TOL and rel_l2 <= REL_L2_TOL, (max_abs, rel_l2)
    return max_abs, rel_l2


def test_c2_full():
    w = workloads.make_inputs("c2")
    out, quant, _ = run_config(w)
    q8, k8, qs, ks = check_quantized(w, quant)
    H, S = w["heads"], w["S"]
    wc = w["words"].numel() // H
    bits = np.stack([oracle.decode_routing(w["words"].numpy()[h * wc:(h + 1) * wc], S, S, 2) for h in range(H)])
    expect = oracle.tilemix_attention(w["q"].numpy(), w["k"].numpy(), w["v"].numpy(), q8, k8, qs, ks,
                                      bits, w["score_scale"], False)
    max_abs, rel_l2 = compare_stats(out.cpu().numpy(), expect)
    assert max_abs <= MAX_ABS_TOL and rel_l2 <= REL_L2_TOL, (max_abs, rel_l2)


def test_c3_full_sampled_rows_and_properties():
    w = workloads.make_inputs("c3")
    out, quant, (q, k, v) = run_config(w)
    quant_host = check_quantized(w, quant)
    heads = np.array([0, 1, 37, 128, 200, 255])
    rows = np.array([0, 1, 2, 15, 16, 63, 64, 127, 128, 129, 511, 1000, 2047, 2048, 3000, 4095])
    sampled_check(w, out, quant_host, heads, rows)
    # all-FP16 mask == unrouted, bit for bit, at full size
    H, S, D = w["heads"], w["S"], w["D"]
    zero = torch.zeros_like(w["words"]).cuda()
    q8, k8, qs, ks = quant
    routed = tm.attention(q, k, v, q8=q8, k8=k8, q_scales=qs, k_scales=ks, words=zero,
                          score_scale=w["score_scale"], causal=True)
    plain = tm.attention(q, k, v, score_scale=w["score_scale"], causal=True)
    torch.cuda.synchronize()
    assert torch.equal(routed.view(torch.int32), plain.view(torch.int32))
    # constant V -> constant O (rows of the softmax sum to one)
    vc = torch.full_like(v, 0.75)
    oc = tm.attention(q, k, vc, q8=q8, k8=k8, q_scales=qs, k_scales=ks, words=w["words"].cuda(),
                      score_scale=w["score_scale"], causal=True)
    torch.cuda.synchronize()
    assert (oc - 0.75).abs().max().item() <= 1e-4   # fp32 accumulation over <= 4096 keys


@pytest.mark.parametrize("p", [0.0, 0.5, 1.0])
def test_c4_long_context_sampled(p):
    w = workloads.make_inputs("c4", p=p)
    out, quant, _ = run_config(w)
    quant_host = check_quantized(w, quant)
    sampled_check(w, out, quant_host, np.array([0, 13, 31]), np.array([0, 127, 4096, 20000, 32767]))


@pytest.mark.parametrize("p", [0.0, 0.25, 0.5, 0.75, 1.0])
def test_c5_routing_sweep_sampled(p):
    w = workloads.make_inputs("c5", p=p)
    out, quant, _ = run_config(w)
    quant_host = check_quantized(w, quant)
    sampled_check(w, out, quant_host, np.array([0, 100, 511]), np.array([0, 63, 64, 700, 1500, 2047]))


@pytest.mark.parametrize("name,p", [("c3", 0.75), ("c3", 0.5), ("c5", 0.5)])
def test_benchmark_inputs_from_the_cuda_generator(name, p):
    """bench.py draws its inputs with the CUDA generator (same distributions,
    different numbers from the CPU one the other tests use); the same
    quantize + attention pass on those exact inputs, checked against the
    oracle: quantization bit-exact on the heads sampled, outputs on sampled
    rows of those heads."""
    w = workloads.make_inputs(name, p=p, device="cuda")
    H, S, D, cfg = w["heads"], w["S"], w["D"], w["cfg"]
    q8, k8, qs, ks = tm.quantize(w["q"], w["k"])
    out = tm.attention(w["q"], w["k"], w["v"], q8=q8, k8=k8, q_scales=qs, k_scales=ks, words=w["words"].cuda(),
                       key_tiles_per_group=2, score_scale=w["score_scale"], causal=cfg["causal"])
    torch.cuda.synchronize()
    err, status = tm.read_and_clear_status()
    assert err == 0 and status == 0
    heads = [0, H // 3, H - 1]
    host = {x: w[x][heads].cpu().numpy() for x in ("q", "k", "v")}
    q8h, k8h, qsh, ksh = (t[heads].cpu().numpy() for t in (q8, k8, qs, ks))
    for i in range(len(heads)):
        eq8, eqs = oracle.quantize(host["q"][i], 128)
        ek8, eks = oracle.quantize(host["k"][i], 64)
        assert np.array_equal(q8h[i], eq8) and np.array_equal(k8h[i], ek8)
        assert np.array_equal(qsh[i].view(np.uint16), eqs.view(np.uint16))
        assert np.array_equal(ksh[i].view(np.uint16), eks.view(np.uint16))
    wc = w["words"].numel() // H
    words = w["words"].numpy()
    bits = np.stack([oracle.decode_routing(words[h * wc:(h + 1) * wc], S, S, 2) for h in heads])
    rows = np.unique(np.concatenate([np.arange(0, S, 97), [S - 1]])).astype(np.int32)
    expect = oracle.tilemix_sampled(host["q"], host["k"], host["v"], q8h, k8h, qsh, ksh, bits,
                                    np.arange(len(heads), dtype=np.int32), rows, w["score_scale"], cfg["causal"])
    actual = out[heads][:, rows].cpu().numpy()
    max_abs, rel_l2 = compare_stats(actual, expect)
    assert max_abs <= MAX_ABS_TOL and rel_l2 <= REL_L2_TOL, (max_abs, rel_l2)
