"""The PyTorch operator layer (torch.ops.tilemix.*) over the C-ABI.

CPU: the operators are registered and their fake kernels give the output
shapes/dtypes (what torch.compile tracing and CUDA-graph capture rely on).
GPU: the operators return exactly what the direct C-ABI calls return.
"""
import math

import numpy as np
import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

from tilemix_b200 import ops  # noqa: F401  (registers torch.ops.tilemix.*)


def test_ops_registered():
    assert hasattr(torch.ops.tilemix, "quantize_qk")
    assert hasattr(torch.ops.tilemix, "attention")
    assert hasattr(torch.ops.tilemix, "attention_bshd")


def test_fake_shapes():
    with FakeTensorMode():
        q = torch.empty((3, 300, 128), dtype=torch.float16)
        k = torch.empty((3, 257, 128), dtype=torch.float16)
        v = torch.empty((3, 257, 128), dtype=torch.float16)
        q8, k8, qs, ks = torch.ops.tilemix.quantize_qk(q, k)
        assert q8.shape == q.shape and q8.dtype == torch.int8
        assert k8.shape == k.shape and k8.dtype == torch.int8
        assert qs.shape == (3, 3) and ks.shape == (3, 5) and qs.dtype == torch.float16
        words = torch.empty((3 * 19,), dtype=torch.int64)
        o = torch.ops.tilemix.attention(q, k, v, q8, k8, qs, ks, words, 2, 0.088, True)
        assert o.shape == q.shape and o.dtype == torch.float32
        o2 = torch.ops.tilemix.attention(q[0], k[0], v[0], None, None, None, None, None, 2, 0.088, False)
        assert o2.shape == (300, 128) and o2.dtype == torch.float32
        o3 = torch.ops.tilemix.attention_bshd(q, k, v, q8, k8, qs, ks, words, 2, 0.088, True, 3, torch.bfloat16)
        assert o3.shape == (1, 300, 3, 128) and o3.dtype == torch.bfloat16


@pytest.mark.gpu
def test_ops_match_c_abi_bitwise():
    import tilemix_b200 as tm
    from tilemix_b200 import workloads
    g = torch.Generator(device="cpu").manual_seed(5)
    heads, m, d = 2, 384, 128
    q = torch.randn((heads, m, d), generator=g).half().cuda()
    k = torch.randn((heads, m, d), generator=g).half().cuda()
    v = torch.randn((heads, m, d), generator=g).half().cuda()
    bm = (torch.rand((heads, (m + 63) // 64, (m + 63) // 64), generator=g) < 0.5).to(torch.uint8).numpy()
    words = torch.from_numpy(workloads.pack_block_mask64(bm, m, m).view(np.int64)).cuda()
    q8, k8, qs, ks = torch.ops.tilemix.quantize_qk(q, k)
    e8, f8, es, fs = tm.quantize(q, k)
    torch.cuda.synchronize()
    assert torch.equal(q8, e8) and torch.equal(k8, f8) and torch.equal(qs, es) and torch.equal(ks, fs)
    scale = 1.0 / math.sqrt(d)
    o = torch.ops.tilemix.attention(q, k, v, q8, k8, qs, ks, words, 2, scale, True)
    e = tm.attention(q, k, v, q8=e8, k8=f8, q_scales=es, k_scales=fs, words=words, key_tiles_per_group=2,
                     score_scale=scale, causal=True)
    torch.cuda.synchronize()
    assert torch.equal(o, e)
    o2 = ops.tilemix_attention(q, k, v, words, causal=True)
    torch.cuda.synchronize()
    assert torch.equal(o2, e)
    err, status = tm.read_and_clear_status()
    assert err == 0 and status == 0


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_attention_bshd_op_is_rounded_default(dtype):
    """torch.ops.tilemix.attention_bshd == the fp32 operator's output, permuted
    to [B, S, H, D] and rounded to the requested type."""
    from tilemix_b200 import workloads
    B, H = 2, 2
    w = workloads.make_inputs("c3", batch=B, heads=H, seq=256)
    q, k, v = (w[n].cuda() for n in ("q", "k", "v"))
    q8, k8, qs, ks = torch.ops.tilemix.quantize_qk(q, k)
    words = w["words"].cuda().view(torch.int64)
    ref = torch.ops.tilemix.attention(q, k, v, q8, k8, qs, ks, words, 2, w["score_scale"], True)
    got = torch.ops.tilemix.attention_bshd(q, k, v, q8, k8, qs, ks, words, 2, w["score_scale"], True, H, dtype)
    assert torch.equal(got, ref.view(B, H, 256, -1).permute(0, 2, 1, 3).to(dtype))


def _meta(shape, dtype=torch.float16):
    return torch.empty(shape, dtype=dtype, device="meta")


@pytest.mark.parametrize("case", [
    "k_heads", "k_dim", "v_shape", "q_dtype", "v_dtype", "q8_shape", "k8_dtype", "q_scales_size",
    "k_scales_size", "words_dtype", "words_short", "words_without_quantized", "partial_quantized", "q_rank"])
def test_validate_rejects_mismatched_tensors(case):
    """The operators and convenience wrappers refuse tensors whose dtype or
    shape disagrees with q's before a device pointer reaches the C-ABI (the
    kernel takes heads and d from q and would read past a smaller tensor)."""
    import tilemix_b200 as tm
    heads, m, n, d = 3, 300, 257, 128
    args = dict(q=_meta((heads, m, d)), k=_meta((heads, n, d)), v=_meta((heads, n, d)),
                q8=_meta((heads, m, d), torch.int8), k8=_meta((heads, n, d), torch.int8),
                q_scales=_meta((heads, 3)), k_scales=_meta((heads, 5)),
                words=_meta((heads * tm.tilemix_routing_word_count(m, n, 2),), torch.int64))
    tm.validate_attention_args(**args, key_tiles_per_group=2, device_check=False)   # the good case passes
    bad = {
        "k_heads": dict(k=_meta((2, n, d)), v=_meta((2, n, d))),
        "k_dim": dict(k=_meta((heads, n, 64)), v=_meta((heads, n, 64))),
        "v_shape": dict(v=_meta((heads, n - 1, d))),
        "q_dtype": dict(q=_meta((heads, m, d), torch.float32)),
        "v_dtype": dict(v=_meta((heads, n, d), torch.bfloat16)),
        "q8_shape": dict(q8=_meta((heads, m - 1, d), torch.int8)),
        "k8_dtype": dict(k8=_meta((heads, n, d), torch.uint8)),
        "q_scales_size": dict(q_scales=_meta((heads, 2))),
        "k_scales_size": dict(k_scales=_meta((heads, 5), torch.float32)),
        "words_dtype": dict(words=_meta((heads * 19,), torch.int32)),
        "words_short": dict(words=_meta((heads * tm.tilemix_routing_word_count(m, n, 2) - 1,), torch.int64)),
        "words_without_quantized": dict(q8=None, k8=None, q_scales=None, k_scales=None),
        "partial_quantized": dict(k8=None, words=None),
        "q_rank": dict(q=_meta((1, heads, m, d))),
    }[case]
    args.update(bad)
    with pytest.raises(ValueError):
        tm.validate_attention_args(**args, key_tiles_per_group=2, device_check=False)


def test_validate_rejects_host_tensors():
    import tilemix_b200 as tm
    q = torch.zeros((2, 64, 64), dtype=torch.float16)
    with pytest.raises(ValueError):
        tm.validate_quantize_args(q, q)
    with pytest.raises(ValueError):
        torch.ops.tilemix.attention(q, q, q, None, None, None, None, None, 2, 0.125, False)


def test_fake_shapes_of_the_newer_operators():
    with FakeTensorMode():
        q = torch.empty((3, 300, 128), dtype=torch.float16)
        k = torch.empty((3, 257, 128), dtype=torch.float16)
        v = torch.empty((3, 257, 128), dtype=torch.float16)
        q8, k8, qs, ks, va = torch.ops.tilemix.quantize_qkv(q, k, v)
        assert va.shape == ks.shape == (3, 5) and va.dtype == torch.float16
        k8b, ks2 = torch.ops.tilemix.quantize_k(k)
        assert k8b.shape == k.shape and ks2.shape == (3, 5)
        words = torch.empty((3 * 19,), dtype=torch.int64)
        o = torch.ops.tilemix.attention_hinted(q, k, v, q8, k8, qs, ks, words, 2, 0.088, True, va)
        assert o.shape == q.shape and o.dtype == torch.float32
        o2, q8f, qsf = torch.ops.tilemix.attention_qfused(q, k, v, k8b, ks2, words, 2, 0.088, True)
        assert o2.shape == q.shape and q8f.shape == q.shape and qsf.shape == (3, 3)
        w = torch.ops.tilemix.routing_policy(qs, ks, 300, 257, 2, 0.5)
        assert w.shape == (3 * 19,) and w.dtype == torch.int64


def test_fake_shapes_of_the_training_operators():
    with FakeTensorMode():
        q = torch.empty((3, 300, 128), dtype=torch.float16)
        k = torch.empty((3, 257, 128), dtype=torch.float16)
        v = torch.empty((3, 257, 128), dtype=torch.float16)
        o, lse = torch.ops.tilemix.attention_lse(q, k, v, 0.088, True)
        assert o.shape == q.shape and o.dtype == torch.float32
        assert lse.shape == (3, 300) and lse.dtype == torch.float32
        do = torch.empty((3, 300, 128), dtype=torch.float16)
        dq, dk, dv = torch.ops.tilemix.attention_backward(q, k, v, o, do, lse, 0.088, True)
        assert dq.shape == q.shape and dk.shape == k.shape and dv.shape == v.shape
        assert dq.dtype == dk.dtype == dv.dtype == torch.float32
        dq2, _, _ = torch.ops.tilemix.attention_backward(q, k, v, o, do, None, 0.088, False)
        assert dq2.shape == q.shape


def test_backward_operator_rejects_bad_tensors_before_the_c_abi():
    q = torch.zeros((2, 64, 64), dtype=torch.float16)
    o = torch.zeros((2, 64, 64), dtype=torch.float32)
    # host tensors (no CUDA device): rejected by the checks, not by a kernel
    with pytest.raises(ValueError):
        torch.ops.tilemix.attention_backward(q, q, q, o, q, None, 0.125, False)
    with pytest.raises(ValueError):
        torch.ops.tilemix.attention_lse(q, q, q, 0.125, False)


@pytest.mark.gpu
def test_newer_operators_match_the_c_abi():
    import tilemix_b200 as tm
    from tilemix_b200 import workloads
    w = workloads.make_inputs("c3", batch=1, heads=2, seq=384)
    q, k, v = (w[x].cuda() for x in ("q", "k", "v"))
    H, S, D = 2, 384, 128
    q8, k8, qs, ks, va = torch.ops.tilemix.quantize_qkv(q, k, v)
    e8, f8, es, fs = tm.quantize(q, k)
    torch.cuda.synchronize()
    assert torch.equal(q8, e8) and torch.equal(k8, f8) and torch.equal(qs, es) and torch.equal(ks, fs)
    words = torch.ops.tilemix.routing_policy(qs, ks, S, S, 2, float(qs.float().median() * ks.float().median()))
    ref_words = torch.empty_like(words)
    assert tm.tilemix_routing_policy(qs, ks, ref_words, H, S, S, 2, float(qs.float().median() * ks.float().median())) == 0
    torch.cuda.synchronize()
    assert torch.equal(words, ref_words)
    expect = tm.attention(q, k, v, q8=q8, k8=k8, q_scales=qs, k_scales=ks, words=words, key_tiles_per_group=2,
                          score_scale=w["score_scale"], causal=True)
    o = torch.ops.tilemix.attention_hinted(q, k, v, q8, k8, qs, ks, words, 2, w["score_scale"], True, va)
    k8b, ksb = torch.ops.tilemix.quantize_k(k)
    o2, q8f, qsf = torch.ops.tilemix.attention_qfused(q, k, v, k8b, ksb, words, 2, w["score_scale"], True)
    torch.cuda.synchronize()
    assert torch.equal(k8b, k8) and torch.equal(ksb, ks) and torch.equal(q8f, q8) and torch.equal(qsf, qs)
    assert torch.equal(o2, expect)
    assert (o - expect).abs().max().item() <= 2e-3      # outlier data: every half two-term, so equal in practice
    err, status = tm.read_and_clear_status()
    assert err == 0 and status == 0
