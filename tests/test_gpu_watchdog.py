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


@pytest.mark.gpu
def test_backward_withheld_arrival_times_out_drains_and_the_next_launch_is_correct():
    """The backward's bounded waits, exercised the same way: its column kernel
    withholds one P-ready arrival per CTA with waits limited to 2 ms."""
    heads, m, d = 2, 512, 128
    g = torch.Generator(device="cpu").manual_seed(13)
    q, k, v, do = (torch.randn((heads, m, d), generator=g).half().cuda() for _ in range(4))
    scale = 1.0 / math.sqrt(d)
    o = torch.empty((heads, m, d), dtype=torch.float32, device="cuda")
    tm.check(tm.tilemix_attention_batched(q, k, v, o, heads, m, m, d, scale), "forward")
    dq, dk, dv = (torch.empty((heads, m, d), dtype=torch.float32, device="cuda") for _ in range(3))
    stats = torch.empty((2, heads, m), dtype=torch.float32, device="cuda")
    assert tm.read_and_clear_status() == (0, 0)

    torch.cuda.synchronize()
    t0 = time.perf_counter()
    assert tm.backward_watchdog_selftest(q, k, v, o, do, dq, dk, dv, stats[0], stats[1], heads, m, m, d, scale,
                                         2000) == 0
    err, status = tm.read_and_clear_status()          # synchronises
    elapsed = time.perf_counter() - t0
    assert err == 0, err
    assert status & tm.STATUS_BACKWARD_WAIT, status
    assert not status & tm.STATUS_BACKWARD_DRAIN, status
    assert status & ~(tm.STATUS_BACKWARD_WAIT | tm.STATUS_BACKWARD_DRAIN) == 0, status
    assert 0.002 <= elapsed < 0.5, elapsed

    # the context is fine: a normal backward on the same stream is correct
    tm.check(tm.tilemix_attention_backward(q, k, v, o, do, dq, dk, dv, stats[0], stats[1], heads, m, m, d, scale),
             "backward")
    torch.cuda.synchronize()
    assert tm.read_and_clear_status() == (0, 0)
    qd, kd, vd = (t.double().requires_grad_() for t in (q, k, v))
    (torch.softmax(scale * qd @ kd.transpose(-1, -2), -1) @ vd).backward(do.double())
    for got, ref in ((dq, qd.grad), (dk, kd.grad), (dv, vd.grad)):
        assert float((got.double() - ref).norm() / ref.norm()) <= 4e-3


def test_backward_selftest_rejects_bad_arguments_without_a_gpu():
    fake = 1 << 20
    args = [fake] * 10 + [1, 128, 128, 128, 0.1]
    assert tm.backward_watchdog_selftest(*args, 0) == tm.cudaErrorInvalidValue
    assert tm.backward_watchdog_selftest(*args, 2_000_000) == tm.cudaErrorInvalidValue
    assert tm.backward_watchdog_selftest(*(args[:13] + [64, 0.1]), 2000) == tm.cudaErrorNotSupported
