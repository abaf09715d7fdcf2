"""The kernel's watchdog, exercised without faulting or hanging the GPU.

Every wait in the attention kernel is bounded. The self-test build withholds
one softmax warp's first "P ready" arrival in every CTA, so the MMA warp of that
key half waits for an arrival that never comes; with a 2 ms limit the wait runs
out, the kernel records the status bit, every role drains its own in-flight TMA
loads and MMAs (a drain that ignores the abort flag) and the CTA returns. The
context stays usable: the next normal launch on the same stream is checked
against the oracle.
"""
import math
import time

import numpy as np
import pytest
import torch

import oracle
import tilemix_b200 as tm


@pytest.mark.gpu
def test_withheld_arrival_times_out_drains_and_the_next_launch_is_correct():
    heads, m, d = 2, 512, 128
    g = torch.Generator(device="cpu").manual_seed(11)
    qh, kh, vh = (torch.randn((heads, m, d), generator=g).half() for _ in range(3))
    q, k, v = qh.cuda(), kh.cuda(), vh.cuda()
    out = torch.empty((heads, m, d), dtype=torch.float32, device="cuda")
    scale = 1.0 / math.sqrt(d)
    err, status = tm.read_and_clear_status()
    assert err == 0 and status == 0, (err, status)

    torch.cuda.synchronize()
    t0 = time.perf_counter()
    assert tm.watchdog_selftest(q, k, v, out, heads, m, m, d, scale, 2000) == 0
    err, status = tm.read_and_clear_status()          # synchronises
    elapsed = time.perf_counter() - t0
    assert err == 0, err
    # a wait ran out (the MMA warp's, or a softmax wait that started at about
    # the same time), and every drain completed within its limit
    assert status & (tm.STATUS_MMA | tm.STATUS_SOFTMAX), status
    assert not status & tm.STATUS_DRAIN, status
    assert status & ~0xF == 0, status
    assert 0.002 <= elapsed < 0.5, elapsed

    # the context is fine: a normal launch on the same stream is correct
    got = tm.attention(q, k, v, score_scale=scale)
    torch.cuda.synchronize()
    err, status = tm.read_and_clear_status()
    assert err == 0 and status == 0, (err, status)
    expect = np.stack([oracle.dense_attention(qh[h].numpy(), kh[h].numpy(), vh[h].numpy()) for h in range(heads)])
    diff = np.abs(got.cpu().numpy().astype(np.float64) - expect)
    assert diff.max() <= 2e-3 and np.linalg.norm(diff) / np.linalg.norm(expect) <= 1e-3


def test_selftest_rejects_bad_limits_without_a_gpu():
    fake = 1 << 20
    assert tm.watchdog_selftest(fake, fake, fake, fake, 1, 128, 128, 128, 0.1, 0) == tm.cudaErrorInvalidValue
    assert tm.watchdog_selftest(fake, fake, fake, fake, 1, 128, 128, 128, 0.1, 2_000_000) == tm.cudaErrorInvalidValue
