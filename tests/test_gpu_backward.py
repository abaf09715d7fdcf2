"""Backward of the unrouted attention on the GPU (no reference counterpart:
the reference is forward only).

The kernels' gradients are compared with float64 autograd of the same formula,
O = softmax(score_scale * Q K^T [causal: key <= query]) V, on the same fp16
Q, K, V and dO. Tolerance: S and dP are fp32 products of fp16 operands, P and
dS enter the second products rounded to fp16 (relative error 2^-11 each), all
accumulation is fp32; and D = rowsum(dO * O) uses the forward kernel's fp32 O.
Each gradient must satisfy
    ||got - ref||_F <= 4e-3 * ||ref||_F   and   max|got - ref| <= 2e-2 * max|ref|.
Outputs are written between guard words that must survive; two runs must be
bit-identical (two launches, no atomics); the watchdog word must stay 0.
"""
import math

import numpy as np
import pytest
import torch

import tilemix_b200 as tm
from tilemix_b200 import ops  # noqa: F401  (registers torch.ops.tilemix.*)

DEV = "cuda:0"
GUARD = -777.5
REL_F, REL_MAX = 4e-3, 2e-2


def reference_grads(q, k, v, do, scale, causal):
    qd, kd, vd = (t.double().requires_grad_() for t in (q, k, v))
    s = scale * qd @ kd.transpose(-1, -2)
    if causal:
        m, n = s.shape[-2:]
        above = torch.arange(n, device=s.device)[None, :] > torch.arange(m, device=s.device)[:, None]
        s = s.masked_fill(above, float("-inf"))
    o = torch.softmax(s, -1) @ vd
    o.backward(do.double())
    return o.detach(), qd.grad, kd.grad, vd.grad


def guarded(shape):
    """fp32 buffer with 4 guard words (16 bytes) on each side; the interior
    keeps the 16-byte alignment the kernels need."""
    count = int(np.prod(shape))
    buf = torch.full((count + 8,), GUARD, dtype=torch.float32, device=DEV)
    return buf, buf[4:-4].view(shape)


def forward(q, k, v, scale, causal):
    heads, m, d = q.shape
    o = torch.empty((heads, m, d), dtype=torch.float32, device=DEV)
    tm.check(tm.tilemix_attention_batched(q, k, v, o, heads, m, k.shape[1], d, scale, causal), "forward")
    return o


def forward_lse(q, k, v, scale, causal):
    heads, m, d = q.shape
    o = torch.empty((heads, m, d), dtype=torch.float32, device=DEV)
    buf, lse = guarded((heads, m))
    tm.check(tm.tilemix_attention_batched_lse(q, k, v, o, lse, heads, m, k.shape[1], d, scale, causal), "forward")
    torch.cuda.synchronize()
    assert torch.all(buf[:4] == GUARD) and torch.all(buf[-4:] == GUARD), "guard overwritten"
    return o, lse


def backward(q, k, v, o, do, scale, causal, lse_in=None):
    heads, m, d = q.shape
    n = k.shape[1]
    bufs = [guarded(s) for s in ((heads, m, d), (heads, n, d), (heads, n, d), (heads, m), (heads, m))]
    dq, dk, dv, lse, dsum = (b[1] for b in bufs)
    if lse_in is not None:
        lse.copy_(lse_in)
    tm.check(tm.tilemix_attention_backward(q, k, v, o, do, dq, dk, dv, lse, dsum, heads, m, n, d, scale, causal,
                                           lse_from_forward=lse_in is not None), "backward")
    torch.cuda.synchronize()
    for buf, _ in bufs:
        assert torch.all(buf[:4] == GUARD) and torch.all(buf[-4:] == GUARD), "guard overwritten"
    return dq, dk, dv, lse, dsum


def inputs(heads, m, n, d, seed, spread=1.0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    q = (spread * torch.randn((heads, m, d), generator=g)).half().to(DEV)
    k = (spread * torch.randn((heads, n, d), generator=g)).half().to(DEV)
    v = torch.randn((heads, n, d), generator=g).half().to(DEV)
    do = torch.randn((heads, m, d), generator=g).half().to(DEV)
    return q, k, v, do


def assert_close(got, ref, name):
    got = got.double()
    err = (got - ref).abs()
    fro = (err.norm() / ref.norm().clamp_min(1e-30)).item()
    mx = (err.max() / ref.abs().max().clamp_min(1e-30)).item()
    assert torch.isfinite(got).all(), f"{name}: non-finite values"
    assert fro <= REL_F and mx <= REL_MAX, f"{name}: relative Frobenius {fro:.2e}, relative max {mx:.2e}"


CASES = [
    # heads, M, N, d, causal
    (2, 256, 256, 64, False),
    (2, 256, 256, 128, False),
    (1, 300, 200, 128, False),     # ragged query and key tiles
    (2, 128, 384, 80, False),      # d not a multiple of 64 (zero-filled atom tail)
    (1, 200, 130, 16, False),      # smallest head dim
    (2, 384, 384, 128, True),
    (1, 200, 450, 64, True),       # keys past the last query: dK = dV = 0 there
    (1, 512, 130, 128, True),      # more queries than keys
    (4, 1024, 1024, 128, True),
    (2, 1024, 2048, 64, False),
]


@pytest.mark.gpu
@pytest.mark.parametrize("heads,m,n,d,causal", CASES)
def test_backward_matches_float64_autograd(heads, m, n, d, causal):
    q, k, v, do = inputs(heads, m, n, d, seed=heads * 1000 + m + n + d + causal)
    scale = 1.0 / math.sqrt(d)
    o = forward(q, k, v, scale, causal)
    o_ref, dq_ref, dk_ref, dv_ref = reference_grads(q, k, v, do, scale, causal)
    dq, dk, dv, lse, dsum = backward(q, k, v, o, do, scale, causal)
    assert_close(dq, dq_ref, "dQ")
    assert_close(dk, dk_ref, "dK")
    assert_close(dv, dv_ref, "dV")
    # the row statistics the launch leaves behind
    s = scale * q.double() @ k.double().transpose(-1, -2)
    if causal:
        above = torch.arange(n, device=DEV)[None, :] > torch.arange(m, device=DEV)[:, None]
        s = s.masked_fill(above, float("-inf"))
    lse_ref = torch.logsumexp(s, -1) / math.log(2.0)
    assert (lse.double() - lse_ref).abs().max().item() <= 1e-3 * max(1.0, lse_ref.abs().max().item())
    dsum_ref = (do.double() * o_ref).sum(-1)
    assert (dsum.double() - dsum_ref).abs().max().item() <= 1e-2 * max(1.0, dsum_ref.abs().max().item())
    if causal and n > m:
        last = ((m - 1) // 128 + 1) * 128          # key tiles no query block sees
        if last < n:
            assert torch.all(dk[:, last:] == 0) and torch.all(dv[:, last:] == 0)
    err, status = tm.read_and_clear_status()
    assert err == 0 and status == 0, (err, status)


@pytest.mark.gpu
def test_backward_is_deterministic():
    heads, m, n, d = 2, 640, 512, 128
    q, k, v, do = inputs(heads, m, n, d, seed=5)
    scale = 0.1
    o = forward(q, k, v, scale, True)
    first = backward(q, k, v, o, do, scale, True)
    second = backward(q, k, v, o, do, scale, True)
    for a, b in zip(first, second):
        assert torch.equal(a.view(torch.int32), b.view(torch.int32))


@pytest.mark.gpu
def test_backward_wide_logits_and_negative_scale():
    # large logit spread (softmax close to one-hot) and a negative score_scale
    heads, m, n, d = 2, 256, 384, 64
    q, k, v, do = inputs(heads, m, n, d, seed=9, spread=3.0)
    for scale in (0.5, -0.125):
        o = forward(q, k, v, scale, False)
        _, dq_ref, dk_ref, dv_ref = reference_grads(q, k, v, do, scale, False)
        dq, dk, dv, _, _ = backward(q, k, v, o, do, scale, False)
        assert_close(dq, dq_ref, f"dQ scale={scale}")
        assert_close(dk, dk_ref, f"dK scale={scale}")
        assert_close(dv, dv_ref, f"dV scale={scale}")


@pytest.mark.gpu
def test_backward_argument_errors():
    q, k, v, do = inputs(1, 128, 128, 64, seed=1)
    o = forward(q, k, v, 0.125, False)
    dq, dk, dv = (torch.empty((1, 128, 64), dtype=torch.float32, device=DEV) for _ in range(3))
    assert tm.tilemix_attention_batched_lse(q, k, v, dq, None, 1, 128, 128, 64, 0.125) == 1
    stats = torch.empty((2, 1, 128), dtype=torch.float32, device=DEV)
    call = tm.tilemix_attention_backward
    assert call(q, k, v, o, None, dq, dk, dv, stats[0], stats[1], 1, 128, 128, 64, 0.125) == 1
    assert call(q, k, v, o, do, dq, dk, dv, stats[0], stats[1], 1, 128, 128, 0, 0.125) == 1
    assert call(q, k, v, o, do, dq, dk, dv, stats[0], stats[1], 1, 128, 128, 64, float("nan")) == 1
    assert call(q, k, v, o, do, dq, dk, dv, stats[0], stats[1], 1, 128, 128, 72, 0.125) == 801   # d % 16
    assert call(q, k, v, o, do, dq, dk, dv, stats[0], stats[1], 1, 128, 128, 144, 0.125) == 801  # d > 128
    flat = torch.empty(128 * 64 + 1, dtype=torch.float32, device=DEV)
    assert call(q, k, v, o, do, flat[1:], dk, dv, stats[0], stats[1], 1, 128, 128, 64, 0.125) == 716
    assert tm.read_and_clear_status() == (0, 0)


@pytest.mark.gpu
def test_autograd_through_the_attention_operator():
    heads, m, n, d = 2, 256, 320, 128
    q, k, v, do = inputs(heads, m, n, d, seed=21)
    scale = 1.0 / math.sqrt(d)
    qg, kg, vg = (t.clone().requires_grad_() for t in (q, k, v))
    out = torch.ops.tilemix.attention(qg, kg, vg, None, None, None, None, None, 2, scale, True)
    out.backward(do.float())
    _, dq_ref, dk_ref, dv_ref = reference_grads(q, k, v, do, scale, True)
    for got, ref, name in ((qg.grad, dq_ref, "dQ"), (kg.grad, dk_ref, "dK"), (vg.grad, dv_ref, "dV")):
        assert got.dtype == torch.float16
        assert_close(got.float(), ref, name)


@pytest.mark.gpu
@pytest.mark.parametrize("heads,m,n,d,causal", [CASES[2], CASES[3], CASES[6], CASES[7], CASES[8]])
def test_backward_from_the_forward_lse(heads, m, n, d, causal):
    q, k, v, do = inputs(heads, m, n, d, seed=heads * 1000 + m + n + d + causal + 7)
    scale = 1.0 / math.sqrt(d)
    o, lse_fwd = forward_lse(q, k, v, scale, causal)
    # the training forward's O is the plain forward's, bit for bit
    assert torch.equal(o.view(torch.int32), forward(q, k, v, scale, causal).view(torch.int32))
    s = scale * q.double() @ k.double().transpose(-1, -2)
    if causal:
        above = torch.arange(n, device=DEV)[None, :] > torch.arange(m, device=DEV)[:, None]
        s = s.masked_fill(above, float("-inf"))
    lse_ref = torch.logsumexp(s, -1) / math.log(2.0)
    assert (lse_fwd.double() - lse_ref).abs().max().item() <= 1e-4 * max(1.0, lse_ref.abs().max().item())
    _, dq_ref, dk_ref, dv_ref = reference_grads(q, k, v, do, scale, causal)
    dq, dk, dv, lse_after, _ = backward(q, k, v, o, do, scale, causal, lse_in=lse_fwd)
    assert torch.equal(lse_after, lse_fwd)        # read, not rewritten
    assert_close(dq, dq_ref, "dQ")
    assert_close(dk, dk_ref, "dK")
    assert_close(dv, dv_ref, "dV")
    assert tm.read_and_clear_status() == (0, 0)


@pytest.mark.gpu
def test_autograd_through_the_training_operator():
    heads, m, n, d = 2, 384, 256, 64
    q, k, v, do = inputs(heads, m, n, d, seed=33)
    scale = 0.2
    qg, kg, vg = (t.clone().requires_grad_() for t in (q, k, v))
    out, lse = torch.ops.tilemix.attention_lse(qg, kg, vg, scale, False)
    out.backward(do.float())
    _, dq_ref, dk_ref, dv_ref = reference_grads(q, k, v, do, scale, False)
    for got, ref, name in ((qg.grad, dq_ref, "dQ"), (kg.grad, dk_ref, "dK"), (vg.grad, dv_ref, "dV")):
        assert got.dtype == torch.float16
        assert_close(got.float(), ref, name)


@pytest.mark.gpu
def test_backward_at_config3_sequence_length():
    """Two heads at config 3's S = 4096, d = 128, causal, from the forward's
    LSE (the training path bench.py --op backward measures), against float64
    autograd: the accumulations run over 32 key or query blocks here."""
    heads, m, n, d = 2, 4096, 4096, 128
    q, k, v, do = inputs(heads, m, n, d, seed=4096)
    scale = 1.0 / math.sqrt(d)
    o, lse_fwd = forward_lse(q, k, v, scale, True)
    _, dq_ref, dk_ref, dv_ref = reference_grads(q, k, v, do, scale, True)
    dq, dk, dv, _, _ = backward(q, k, v, o, do, scale, True, lse_in=lse_fwd)
    assert_close(dq, dq_ref, "dQ")
    assert_close(dk, dk_ref, "dK")
    assert_close(dv, dv_ref, "dV")
    assert tm.read_and_clear_status() == (0, 0)


EDGE_CASES = [
    # heads, M, N, d, causal, score_scale (None: 1/sqrt(d))
    (2, 200, 300, 32, False, None),
    (1, 130, 257, 48, True, None),
    (2, 256, 192, 96, False, None),
    (1, 300, 300, 112, True, None),
    (1, 1, 1, 64, False, None),        # one query, one key: P = 1, dS = 0
    (1, 1, 700, 128, False, None),     # one query row against a long key range
    (1, 700, 1, 64, True, None),       # one key, causal: every row sees only key 0
    (2, 256, 256, 64, False, 0.0),     # score_scale 0: uniform softmax, dQ = dK = 0
]


@pytest.mark.gpu
@pytest.mark.parametrize("heads,m,n,d,causal,scale", EDGE_CASES)
def test_backward_edge_cases(heads, m, n, d, causal, scale):
    q, k, v, do = inputs(heads, m, n, d, seed=heads * 7 + m * 3 + n + d)
    scale = 1.0 / math.sqrt(d) if scale is None else scale
    o = forward(q, k, v, scale, causal)
    _, dq_ref, dk_ref, dv_ref = reference_grads(q, k, v, do, scale, causal)
    dq, dk, dv, _, _ = backward(q, k, v, o, do, scale, causal)
    for got, ref, name in ((dq, dq_ref, "dQ"), (dk, dk_ref, "dK"), (dv, dv_ref, "dV")):
        if float(ref.abs().max()) < 1e-12:
            # an exactly-zero gradient (one key, or score_scale 0) must come out as (near) zero
            assert float(got.abs().max()) <= 1e-5, (name, float(got.abs().max()))
        else:
            assert_close(got, ref, name)
    assert tm.read_and_clear_status() == (0, 0)
