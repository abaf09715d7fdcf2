"""GPU: the pipelined host-buffer entry point (tilemix_attention_from_host)
gives exactly the device-buffer path's results (same kernels, same inputs:
bit-for-bit) for every chunking, routed and unrouted, causal and not, and its
routed output matches the CPU oracle within the parity tolerance."""
import math

import numpy as np
import pytest
import torch

import oracle
from refcases import MAX_ABS_TOL, REL_L2_TOL, compare_stats
import tilemix_b200 as tm
from tilemix_b200 import workloads

pytestmark = pytest.mark.gpu


def device_path(w, causal, routed):
    q, k, v = (w[n].cuda() for n in ("q", "k", "v"))
    heads, S, D = w["heads"], w["S"], w["D"]
    if routed:
        q8, k8, qs, ks = tm.quantize(q, k)
        out = tm.attention(q, k, v, q8=q8, k8=k8, q_scales=qs, k_scales=ks, words=w["words"].cuda(),
                           key_tiles_per_group=2, causal=causal)
        return out.cpu(), (q8.cpu(), k8.cpu(), qs.cpu(), ks.cpu())
    return tm.attention(q, k, v, causal=causal).cpu(), None


def host_path(w, causal, routed, chunk, stream=None):
    heads, S, D = w["heads"], w["S"], w["D"]
    hq, hk, hv = (w[n].pin_memory() for n in ("q", "k", "v"))
    hw = w["words"].pin_memory() if routed else None
    ho = torch.full((heads, S, D), float("nan"), dtype=torch.float32).pin_memory()
    bufs = tm.TileMixDeviceBuffers(
        q=torch.empty_like(hq, device="cuda"), k=torch.empty_like(hk, device="cuda"),
        v=torch.empty_like(hv, device="cuda"), o=torch.empty((heads, S, D), dtype=torch.float32, device="cuda"))
    if routed:
        bufs.q8 = torch.empty((heads, S, D), dtype=torch.int8, device="cuda")
        bufs.k8 = torch.empty((heads, S, D), dtype=torch.int8, device="cuda")
        bufs.q_scales = torch.empty((heads, (S - 1) // 128 + 1), dtype=torch.float16, device="cuda")
        bufs.k_scales = torch.empty((heads, (S - 1) // 64 + 1), dtype=torch.float16, device="cuda")
        bufs.words = torch.empty_like(hw, device="cuda")
    err = tm.tilemix_attention_from_host(hq, hk, hv, hw, ho, bufs, heads, S, S, D, w["score_scale"],
                                         causal, 2, chunk, stream)
    assert err == 0, err
    if stream is not None:
        stream.synchronize()       # the call's completion is ordered on its stream
    else:
        torch.cuda.current_stream().synchronize()
    quant = (bufs.q8.cpu(), bufs.k8.cpu(), bufs.q_scales.cpu(), bufs.k_scales.cpu()) if routed else None
    return ho.clone(), quant


@pytest.mark.parametrize("name,heads,seq,causal,routed,chunk", [
    ("c2", 6, 384, False, True, 0),
    ("c2", 6, 384, False, True, 1),
    ("c2", 6, 384, True, True, 4),
    ("c3", 5, 700, True, True, 2),
    ("c3", 3, 256, True, False, 0),
    ("c5", 4, 512, True, True, 16),
])
def test_from_host_equals_device_path(name, heads, seq, causal, routed, chunk):
    w = workloads.make_inputs(name, batch=1, heads=heads, seq=seq)
    expect, q_dev = device_path(w, causal, routed)
    got, q_host = host_path(w, causal, routed, chunk, stream=torch.cuda.Stream())
    assert torch.equal(got, expect)
    if routed:
        for a, b in zip(q_host, q_dev):
            assert torch.equal(a, b)
    err, status = tm.read_and_clear_status()
    assert err == 0 and status == 0


def test_from_host_matches_oracle():
    w = workloads.make_inputs("c3", batch=1, heads=2, seq=512)
    got, (q8, k8, qs, ks) = host_path(w, True, True, 1)
    S = w["S"]
    q, k, v = (w[n].numpy() for n in ("q", "k", "v"))
    eq8, eqs = oracle.quantize(q, 128)
    ek8, eks = oracle.quantize(k, 64)
    assert np.array_equal(q8.numpy(), eq8) and np.array_equal(k8.numpy(), ek8)
    assert np.array_equal(qs.numpy().view(np.uint16), eqs.view(np.uint16))
    assert np.array_equal(ks.numpy().view(np.uint16), eks.view(np.uint16))
    wc = w["words"].numel() // 2
    words = w["words"].numpy()
    bits = np.stack([oracle.decode_routing(words[h * wc:(h + 1) * wc], S, S, 2) for h in range(2)])
    expect = oracle.tilemix_attention(q, k, v, eq8, ek8, eqs, eks, bits, 1.0 / math.sqrt(w["D"]), causal=True)
    max_abs, rel_l2 = compare_stats(got.numpy(), expect)
    assert max_abs <= MAX_ABS_TOL and rel_l2 <= REL_L2_TOL, (max_abs, rel_l2)
