"""GPU: accuracy beside the reference's own GPU kernel on config 3's data.

Config 3 scales 1 % of the head-dim channels by 20 in Q, K and V, so an FP16
score q.k reaches thousands and the tensor core's fp32 accumulation of the
fp16 products (16 per MMA step, in hardware order) carries errors that the
fp64 oracle does not have. The reference's GPU kernel (src/tilemix.cu: WMMA
fp16 x fp16 -> fp32 for FP16 tiles, INT8 WMMA for INT8 tiles) meets the same
limit. This test runs both kernels on the first heads of the benchmark's own
inputs (CUDA generator, config 3's seed) and checks that, per head, ours stays
inside the parity bar or within 25 % of the reference kernel's own max-abs
error, with the relative-L2 bar met. The reference kernel has no causal mask,
so the heads run non-causal. Skipped when oracle/_ref holds no GPU build of
the reference.
"""
import math

import numpy as np
import pytest
import torch

import oracle
from refcases import MAX_ABS_TOL, REL_L2_TOL
import tilemix_b200 as tm
from tilemix_b200 import workloads

pytestmark = pytest.mark.gpu

HEADS = 6


def test_config3_error_matches_reference_gpu_kernel():
    lib = oracle.ref_gpu_lib()
    if lib is None:
        pytest.skip("no GPU build of the reference under oracle/_ref")
    w = workloads.make_inputs("c3", batch=1, heads=256, seed=workloads.config("c3")["seed"], device="cuda")
    H, S, D = w["heads"], w["S"], w["D"]
    q, k, v = (w[x][:HEADS].contiguous() for x in ("q", "k", "v"))
    wc = w["words"].numel() // H
    words_host = w["words"].numpy()[:HEADS * wc].copy()
    words = torch.from_numpy(words_host).cuda()
    q8, k8, qs, ks = tm.quantize(q, k)
    ours = tm.attention(q, k, v, q8=q8, k8=k8, q_scales=qs, k_scales=ks, words=words, key_tiles_per_group=2,
                        score_scale=w["score_scale"], causal=False)
    theirs = torch.empty((HEADS, S, D), dtype=torch.float32, device="cuda")
    q8r, k8r, qsr, ksr = (torch.empty_like(t) for t in (q8, k8, qs, ks))
    rc = lib.ref_gpu_tilemix_heads(q.data_ptr(), k.data_ptr(), v.data_ptr(), q8r.data_ptr(), k8r.data_ptr(),
                                   qsr.data_ptr(), ksr.data_ptr(), theirs.data_ptr(), HEADS, S, S, D,
                                   w["score_scale"], words.data_ptr(), wc, 2, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert rc == 0
    err, status = tm.read_and_clear_status()
    assert err == 0 and status == 0
    # same quantized bytes as the reference's own quantizer
    assert torch.equal(q8, q8r) and torch.equal(k8, k8r) and torch.equal(qs, qsr) and torch.equal(ks, ksr)
    hq, hk, hv = (t.cpu().numpy() for t in (q, k, v))
    h8q, h8k, hqs, hks = (t.cpu().numpy() for t in (q8, k8, qs, ks))
    go, gt = ours.cpu().numpy(), theirs.cpu().numpy()
    for h in range(HEADS):
        bits = oracle.decode_routing(words_host[h * wc:(h + 1) * wc], S, S, 2)[None]
        ref = oracle.tilemix_sampled(hq[h:h + 1], hk[h:h + 1], hv[h:h + 1], h8q[h:h + 1], h8k[h:h + 1],
                                     hqs[h:h + 1], hks[h:h + 1], bits, np.array([0], np.int32),
                                     np.arange(S, dtype=np.int32), 1.0 / math.sqrt(D), False)[0]
        e_ours = np.abs(go[h].astype(np.float64) - ref)
        e_ref = np.abs(gt[h].astype(np.float64) - ref)
        rel_ours = float(np.linalg.norm(e_ours) / np.linalg.norm(ref))
        assert rel_ours <= REL_L2_TOL, (h, rel_ours)
        assert e_ours.max() <= max(MAX_ABS_TOL, 1.25 * e_ref.max()), (h, float(e_ours.max()), float(e_ref.max()))
