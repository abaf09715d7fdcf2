"""The device routing policy (tilemix_routing_policy) and its CPU restatement.

Policy: a (16-row query tile, key group) pair is INT8 iff
fl32(q_scale * max k_scale over the group's 64-row K blocks) <= max_product;
outlier blocks stay FP16. Words use the reference's mask format
(src/tilemix.cu:99-103).

CPU: the oracle's C restatement equals an independent pure-Python loop.
GPU: the kernel's words equal the oracle's bit for bit (ragged shapes, every
group size, NaN / inf / zero scales), and attention with policy-chosen masks
matches the oracle within the parity tolerance.
"""
import math

import numpy as np
import pytest
import torch

import oracle
import refcases

INT_MAX = 2**31 - 1
SHAPES = [(300, 1000, 2, 2), (17, 4099, 3, 1), (129, 131, 1, 3), (1, 1, 1, 1), (17, 65, INT_MAX, 2),
          (4096, 4096, 2, 2), (1000, 1003, 5, 1), (256, 8192, 64, 1)]


def _scales(rng, heads, blocks):
    return (rng.uniform(0.001, 1.0, (heads, blocks)) * rng.choice([1.0, 20.0], (heads, blocks))).astype(np.float16)


def _python_policy(qs, ks, heads, m, n, g, t):
    q16, k32 = -(-m // 16), -(-n // 32)
    groups = -(-k32 // g)
    wpr = -(-groups // 64)
    out = np.zeros(heads * q16 * wpr, np.uint64)
    for h in range(heads):
        for tile in range(q16):
            sq = np.float32(qs[h, tile // 8])
            for gr in range(groups):
                key0 = gr * g * 32
                key1 = min(min(gr * g + g, k32) * 32, n)
                blocks = ks[h, key0 // 64:(key1 - 1) // 64 + 1].astype(np.float32)
                if np.isnan(blocks).any():
                    continue
                if np.float32(sq * np.float32(blocks.max())) <= np.float32(t):
                    out[(h * q16 + tile) * wpr + gr // 64] |= np.uint64(1) << np.uint64(gr % 64)
    return out


def _thresholds_with_specials(rng, qs, ks):
    """Plants a NaN, an inf and a zero scale (where there is more than one
    scale) and returns thresholds spanning all-FP16 to all-INT8."""
    qf, kf = qs.astype(np.float32).reshape(-1), ks.astype(np.float32).reshape(-1)
    ts = [0.0, float(np.quantile(qf.max() * kf, 1 / 3)), float(np.median(qf) * np.median(kf)), 3.0e38]
    if ks.size > 1:
        ks.reshape(-1)[rng.integers(0, ks.size)] = np.nan
        ks.reshape(-1)[rng.integers(0, ks.size)] = 0
    if qs.size > 1:
        qs.reshape(-1)[rng.integers(0, qs.size)] = np.inf
    return ts


@pytest.mark.parametrize("m,n,g,heads", [s for s in SHAPES if s[0] * s[1] <= 4_000_000 and s[2] < 1000])
def test_oracle_policy_matches_a_python_restatement(m, n, g, heads):
    rng = np.random.default_rng(m + n + g)
    qs, ks = _scales(rng, heads, -(-m // 128)), _scales(rng, heads, -(-n // 64))
    ks[0, 0] = np.nan
    t = float(np.median(qs.astype(np.float32)) * np.median(ks.astype(np.float32)))
    assert np.array_equal(oracle.routing_policy(qs, ks, heads, m, n, g, t), _python_policy(qs, ks, heads, m, n, g, t))


def test_threshold_cases_are_finite():
    for m, n, g, heads in SHAPES:
        rng = np.random.default_rng(m * 3 + n + heads)
        qs, ks = _scales(rng, heads, -(-m // 128)), _scales(rng, heads, -(-n // 64))
        assert all(np.isfinite(t) for t in _thresholds_with_specials(rng, qs, ks))


@pytest.mark.gpu
@pytest.mark.parametrize("m,n,g,heads", SHAPES)
def test_gpu_policy_words_bit_exact(m, n, g, heads):
    import tilemix_b200 as tm
    rng = np.random.default_rng(m * 3 + n + heads)
    qs, ks = _scales(rng, heads, -(-m // 128)), _scales(rng, heads, -(-n // 64))
    wc = tm.tilemix_routing_word_count(m, n, g)
    for t in _thresholds_with_specials(rng, qs, ks):
        words = torch.full((heads * wc + 2,), 0x5A5A5A5A5A5A5A5A, dtype=torch.int64, device="cuda")
        assert tm.tilemix_routing_policy(torch.from_numpy(qs).cuda(), torch.from_numpy(ks).cuda(), words[1:-1], heads,
                                         m, n, g, t) == 0
        got = words.cpu().numpy().view(np.uint64)
        assert got[0] == got[-1] == np.uint64(0x5A5A5A5A5A5A5A5A), "guard overwritten"
        assert np.array_equal(got[1:-1], oracle.routing_policy(qs, ks, heads, m, n, g, t)), t


@pytest.mark.gpu
def test_attention_with_policy_masks_matches_the_oracle():
    """Quantize -> policy -> attention on a config-3 shape (outlier channels,
    causal): the policy's words drive the kernel and the oracle alike."""
    import tilemix_b200 as tm
    from tilemix_b200 import workloads
    w = workloads.make_inputs("c3", batch=1, heads=3, seq=1024)
    H, S, D = w["heads"], w["S"], w["D"]
    q, k, v = (w[x].cuda() for x in ("q", "k", "v"))
    q8, k8, qs, ks = tm.quantize(q, k)
    torch.cuda.synchronize()
    qf, kf = qs.cpu().float().numpy(), ks.cpu().float().numpy()
    t = float(np.median(qf[:, :, None] * kf[:, None, :]))      # about half the tiles INT8
    words = torch.empty(H * tm.tilemix_routing_word_count(S, S, 2), dtype=torch.int64, device="cuda")
    assert tm.tilemix_routing_policy(qs, ks, words, H, S, S, 2, t) == 0
    out = tm.attention(q, k, v, q8=q8, k8=k8, q_scales=qs, k_scales=ks, words=words, key_tiles_per_group=2,
                       score_scale=w["score_scale"], causal=True)
    torch.cuda.synchronize()
    host_words = words.cpu().numpy().view(np.uint64)
    assert np.array_equal(host_words, oracle.routing_policy(qs.cpu().numpy(), ks.cpu().numpy(), H, S, S, 2, t))
    wc = host_words.size // H
    bits = np.stack([oracle.decode_routing(host_words[h * wc:(h + 1) * wc], S, S, 2) for h in range(H)])
    frac = float(bits.mean())
    assert 0.05 < frac < 0.95, frac          # a real mix of INT8 and FP16 tiles
    rows = np.arange(0, S, 7, dtype=np.int32)
    qh, kh, vh = (w[x].numpy() for x in ("q", "k", "v"))
    expect = oracle.tilemix_sampled(qh, kh, vh, q8.cpu().numpy(), k8.cpu().numpy(), qs.cpu().numpy(),
                                    ks.cpu().numpy(), bits, np.arange(H, dtype=np.int32), rows, w["score_scale"], True)
    got = out.cpu().numpy()[:, rows].astype(np.float64)
    diff = np.abs(got - expect)
    assert diff.max() <= refcases.MAX_ABS_TOL and np.linalg.norm(diff) / np.linalg.norm(expect) <= 1e-3


def test_threshold_helper():
    import tilemix_b200 as tm
    t = tm.tilemix_policy_max_scale_product(0.5, 1 / math.sqrt(128), 128)
    assert abs(t - 0.5 / (128 ** -0.5 * 128 * 127.25)) < 1e-9
    assert tm.tilemix_policy_max_scale_product(0.5, 0.0, 128) > 1e38
