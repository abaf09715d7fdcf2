"""PyTorch operators over the C-ABI: ``torch.ops.tilemix.quantize_qk``,
``.attention``, ``.attention_bshd``, ``.quantize_qkv`` + ``.attention_hinted``
(single-term P from V statistics), ``.quantize_k`` + ``.attention_qfused`` (Q
quantized inside the kernel), ``.routing_policy`` (routing words chosen on
the device), ``.attention_backward`` (gradients of the unrouted attention,
registered as the autograd formula of ``.attention``) and ``.attention_lse``
(the training forward: output and row log-sum-exp, whose autograd formula
reuses the saved statistics).

They call the same extern "C" entry points as the ctypes functions in
``tilemix_b200`` (``tilemix_quantize_qk_batched``, ``tilemix_attention_batched``)
on the current CUDA stream, and register fake (meta) kernels so that shape
propagation, ``torch.compile`` tracing and CUDA-graph capture see the outputs
without running the GPU code. Every operator checks dtypes, devices and
cross-tensor shapes (``validate_attention_args``) before a device pointer
reaches the C-ABI. Layout: [heads, S, d] contiguous fp16 (a 2-D
[S, d] tensor is one head), the reference's layout per head; the routing words
are the reference's per-head mask words (``include/attention_fused.h:47-52``),
``words_per_head`` apart.
"""
from __future__ import annotations

import math

import torch

from . import (TileMixOutput, TileMixQuantized, TileMixRouting, _require, check, quantize_tilemix_k_batched,
               quantize_tilemix_qk_batched, quantize_tilemix_qkv_batched, tilemix_attention_batched,
               tilemix_attention_backward, tilemix_attention_batched_hinted, tilemix_attention_batched_lse, tilemix_attention_batched_out,
               tilemix_attention_batched_qfused,
               tilemix_routing_policy, tilemix_routing_word_count, validate_attention_args, validate_quantize_args)

_Q_ROWS, _K_ROWS = 128, 64   # quantization block rows (include/attention_fused.h:13-14)


def _heads3(x: torch.Tensor) -> torch.Tensor:
    return x if x.dim() == 3 else x.unsqueeze(0)


def _contiguous(*ts):
    return tuple(None if t is None else t.contiguous() for t in ts)


@torch.library.custom_op("tilemix::quantize_qk", mutates_args=())
def quantize_qk(q: torch.Tensor, k: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """Per-block symmetric INT8 quantization of Q (128-row blocks) and K (64-row
    blocks): returns (q8, k8, q_scales [heads, ceil(M/128)], k_scales [heads, ceil(N/64)])."""
    heads, m, n, d = validate_quantize_args(q, k)
    q3, k3 = _heads3(q).contiguous(), _heads3(k).contiguous()
    q8 = torch.empty(q.shape, dtype=torch.int8, device=q.device)
    k8 = torch.empty(k.shape, dtype=torch.int8, device=k.device)
    qs = torch.empty((heads, (m - 1) // _Q_ROWS + 1), dtype=torch.float16, device=q.device)
    ks = torch.empty((heads, (n - 1) // _K_ROWS + 1), dtype=torch.float16, device=q.device)
    check(quantize_tilemix_qk_batched(q3, k3, q8, k8, qs, ks, heads, m, n, d,
                                      torch.cuda.current_stream(q.device)), "tilemix::quantize_qk")
    return q8, k8, qs, ks


@quantize_qk.register_fake
def _(q, k):
    heads = 1 if q.dim() == 2 else q.shape[0]
    m, n = q.shape[-2], k.shape[-2]
    return (q.new_empty(q.shape, dtype=torch.int8), k.new_empty(k.shape, dtype=torch.int8),
            q.new_empty((heads, (m - 1) // _Q_ROWS + 1), dtype=torch.float16),
            q.new_empty((heads, (n - 1) // _K_ROWS + 1), dtype=torch.float16))


@torch.library.custom_op("tilemix::attention", mutates_args=())
def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, q8: torch.Tensor | None,
              k8: torch.Tensor | None, q_scales: torch.Tensor | None, k_scales: torch.Tensor | None,
              words: torch.Tensor | None, key_tiles_per_group: int, score_scale: float,
              causal: bool) -> torch.Tensor:
    """Routed mixed-precision attention, fp32 output of q's shape. With
    ``words`` (uint64 mask words viewed as int64) the quantized operands are
    required; without, every tile runs FP16 (the reference's unrouted path)."""
    heads, m, n, d = validate_attention_args(q, k, v, q8, k8, q_scales, k_scales, words, key_tiles_per_group)
    q3, k3, v3 = _heads3(q).contiguous(), _heads3(k).contiguous(), _heads3(v).contiguous()
    q8, k8, q_scales, k_scales, words = _contiguous(q8, k8, q_scales, k_scales, words)
    out = torch.empty(q.shape, dtype=torch.float32, device=q.device)
    routing = TileMixRouting(words, 0 if words is None else words.numel(), key_tiles_per_group)
    quantized = TileMixQuantized(q8, k8, q_scales, k_scales) if q8 is not None else None
    check(tilemix_attention_batched(q3, k3, v3, out, heads, m, n, d, score_scale, causal,
                                    torch.cuda.current_stream(q.device), routing, quantized),
          "tilemix::attention")
    return out


@attention.register_fake
def _(q, k, v, q8, k8, q_scales, k_scales, words, key_tiles_per_group, score_scale, causal):
    return q.new_empty(q.shape, dtype=torch.float32)


@torch.library.custom_op("tilemix::attention_bshd", mutates_args=())
def attention_bshd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, q8: torch.Tensor | None,
                   k8: torch.Tensor | None, q_scales: torch.Tensor | None, k_scales: torch.Tensor | None,
                   words: torch.Tensor | None, key_tiles_per_group: int, score_scale: float, causal: bool,
                   heads_per_batch: int, out_dtype: torch.dtype) -> torch.Tensor:
    """``attention`` with the output written by the kernel as [B, S, H, D]
    (heads = B * H of q's [heads, S, d]) in fp32, fp16 or bf16 (rounded to
    nearest even from the fp32 result)."""
    heads, m, n, d = validate_attention_args(q, k, v, q8, k8, q_scales, k_scales, words, key_tiles_per_group)
    q3, k3, v3 = _heads3(q).contiguous(), _heads3(k).contiguous(), _heads3(v).contiguous()
    q8, k8, q_scales, k_scales, words = _contiguous(q8, k8, q_scales, k_scales, words)
    if heads_per_batch < 1 or heads % heads_per_batch:
        raise ValueError(f"heads_per_batch {heads_per_batch} must divide the {heads} heads")
    if out_dtype not in (torch.float32, torch.float16, torch.bfloat16):
        raise ValueError(f"out_dtype must be float32, float16 or bfloat16, got {out_dtype}")
    out = torch.empty((heads // heads_per_batch, m, heads_per_batch, d), dtype=out_dtype, device=q.device)
    routing = TileMixRouting(words, 0 if words is None else words.numel(), key_tiles_per_group)
    quantized = TileMixQuantized(q8, k8, q_scales, k_scales) if q8 is not None else None
    check(tilemix_attention_batched_out(q3, k3, v3, TileMixOutput.bshd(out, heads_per_batch), heads, m, n, d,
                                        score_scale, causal, torch.cuda.current_stream(q.device), routing,
                                        quantized), "tilemix::attention_bshd")
    return out


@attention_bshd.register_fake
def _(q, k, v, q8, k8, q_scales, k_scales, words, key_tiles_per_group, score_scale, causal, heads_per_batch,
      out_dtype):
    heads = 1 if q.dim() == 2 else q.shape[0]
    return q.new_empty((heads // heads_per_batch, q.shape[-2], heads_per_batch, q.shape[-1]), dtype=out_dtype)


@torch.library.custom_op("tilemix::quantize_qkv", mutates_args=())
def quantize_qkv(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor,
                                                                          torch.Tensor, torch.Tensor]:
    """quantize_qk plus max |v| per 64-row block of V (fp16 [heads, ceil(N/64)]),
    the statistics attention_hinted uses for single-term P."""
    heads, m, n, d = validate_attention_args(q, k, v)
    q3, k3, v3 = _heads3(q).contiguous(), _heads3(k).contiguous(), _heads3(v).contiguous()
    q8 = torch.empty(q.shape, dtype=torch.int8, device=q.device)
    k8 = torch.empty(k.shape, dtype=torch.int8, device=k.device)
    qs = torch.empty((heads, (m - 1) // _Q_ROWS + 1), dtype=torch.float16, device=q.device)
    ks = torch.empty((heads, (n - 1) // _K_ROWS + 1), dtype=torch.float16, device=q.device)
    va = torch.empty((heads, (n - 1) // _K_ROWS + 1), dtype=torch.float16, device=q.device)
    check(quantize_tilemix_qkv_batched(q3, k3, v3, q8, k8, qs, ks, va, heads, m, n, d,
                                       torch.cuda.current_stream(q.device)), "tilemix::quantize_qkv")
    return q8, k8, qs, ks, va


@quantize_qkv.register_fake
def _(q, k, v):
    heads = 1 if q.dim() == 2 else q.shape[0]
    m, n = q.shape[-2], k.shape[-2]
    kb = (n - 1) // _K_ROWS + 1
    return (q.new_empty(q.shape, dtype=torch.int8), k.new_empty(k.shape, dtype=torch.int8),
            q.new_empty((heads, (m - 1) // _Q_ROWS + 1), dtype=torch.float16),
            q.new_empty((heads, kb), dtype=torch.float16), q.new_empty((heads, kb), dtype=torch.float16))


@torch.library.custom_op("tilemix::attention_hinted", mutates_args=())
def attention_hinted(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, q8: torch.Tensor | None,
                     k8: torch.Tensor | None, q_scales: torch.Tensor | None, k_scales: torch.Tensor | None,
                     words: torch.Tensor | None, key_tiles_per_group: int, score_scale: float, causal: bool,
                     v_absmax: torch.Tensor) -> torch.Tensor:
    """``attention`` with single-term fp16 P for the 64-key halves whose max |v|
    (``v_absmax`` from quantize_qkv) is <= 3.5 (at most 1.7e-3 added to any output)."""
    heads, m, n, d = validate_attention_args(q, k, v, q8, k8, q_scales, k_scales, words, key_tiles_per_group)
    if v_absmax.dtype != torch.float16 or v_absmax.numel() != heads * ((n - 1) // _K_ROWS + 1) or \
            v_absmax.device != q.device:
        raise ValueError("v_absmax must be fp16 [heads, ceil(N/64)] on q's device")
    q3, k3, v3 = _heads3(q).contiguous(), _heads3(k).contiguous(), _heads3(v).contiguous()
    q8, k8, q_scales, k_scales, words, v_absmax = _contiguous(q8, k8, q_scales, k_scales, words, v_absmax)
    out = torch.empty(q.shape, dtype=torch.float32, device=q.device)
    routing = TileMixRouting(words, 0 if words is None else words.numel(), key_tiles_per_group)
    quantized = TileMixQuantized(q8, k8, q_scales, k_scales) if q8 is not None else None
    check(tilemix_attention_batched_hinted(q3, k3, v3, out, heads, m, n, d, score_scale, causal,
                                           torch.cuda.current_stream(q.device), routing, quantized, v_absmax),
          "tilemix::attention_hinted")
    return out


@attention_hinted.register_fake
def _(q, k, v, q8, k8, q_scales, k_scales, words, key_tiles_per_group, score_scale, causal, v_absmax):
    return q.new_empty(q.shape, dtype=torch.float32)


@torch.library.custom_op("tilemix::quantize_k", mutates_args=())
def quantize_k(k: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """K alone in 64-row blocks (the pre-pass of attention_qfused)."""
    heads, _, n, d = validate_quantize_args(k, k)
    k3 = _heads3(k).contiguous()
    k8 = torch.empty(k.shape, dtype=torch.int8, device=k.device)
    ks = torch.empty((heads, (n - 1) // _K_ROWS + 1), dtype=torch.float16, device=k.device)
    check(quantize_tilemix_k_batched(k3, k8, ks, heads, n, d, torch.cuda.current_stream(k.device)),
          "tilemix::quantize_k")
    return k8, ks


@quantize_k.register_fake
def _(k):
    heads = 1 if k.dim() == 2 else k.shape[0]
    return (k.new_empty(k.shape, dtype=torch.int8),
            k.new_empty((heads, (k.shape[-2] - 1) // _K_ROWS + 1), dtype=torch.float16))


@torch.library.custom_op("tilemix::attention_qfused", mutates_args=())
def attention_qfused(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, k8: torch.Tensor, k_scales: torch.Tensor,
                     words: torch.Tensor, key_tiles_per_group: int, score_scale: float,
                     causal: bool) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Routed attention that quantizes each 128-row Q tile inside the kernel;
    returns (out, q8, q_scales), q8 / q_scales the bytes quantize_qk makes."""
    heads, m, n, d = validate_attention_args(q, k, v, words=None)
    if k8.dtype != torch.int8 or tuple(k8.shape) != tuple(k.shape) or k_scales.dtype != torch.float16 or \
            k_scales.numel() != heads * ((n - 1) // _K_ROWS + 1):
        raise ValueError("k8 / k_scales must come from quantize_k on this k")
    if words.dtype not in (torch.int64, torch.uint64) or \
            words.numel() < heads * tilemix_routing_word_count(m, n, key_tiles_per_group):
        raise ValueError("words must be 64-bit and hold heads * tilemix_routing_word_count words")
    q3, k3, v3 = _heads3(q).contiguous(), _heads3(k).contiguous(), _heads3(v).contiguous()
    k8, k_scales, words = _contiguous(k8, k_scales, words)
    out = torch.empty(q.shape, dtype=torch.float32, device=q.device)
    q8 = torch.empty(q.shape, dtype=torch.int8, device=q.device)
    qs = torch.empty((heads, (m - 1) // _Q_ROWS + 1), dtype=torch.float16, device=q.device)
    check(tilemix_attention_batched_qfused(q3, k3, v3, out, heads, m, n, d, score_scale, causal,
                                           torch.cuda.current_stream(q.device),
                                           TileMixRouting(words, words.numel(), key_tiles_per_group), k8, k_scales,
                                           q8, qs), "tilemix::attention_qfused")
    return out, q8, qs


@attention_qfused.register_fake
def _(q, k, v, k8, k_scales, words, key_tiles_per_group, score_scale, causal):
    heads = 1 if q.dim() == 2 else q.shape[0]
    return (q.new_empty(q.shape, dtype=torch.float32), q.new_empty(q.shape, dtype=torch.int8),
            q.new_empty((heads, (q.shape[-2] - 1) // _Q_ROWS + 1), dtype=torch.float16))


@torch.library.custom_op("tilemix::routing_policy", mutates_args=())
def routing_policy(q_scales: torch.Tensor, k_scales: torch.Tensor, m: int, n: int, key_tiles_per_group: int,
                   max_scale_product: float) -> torch.Tensor:
    """Routing words (int64 view of the reference's uint64 mask words) chosen on
    the device: INT8 iff q_scale * max k_scale of the key group <= max_scale_product."""
    heads = q_scales.shape[0] if q_scales.dim() == 2 else 1
    if q_scales.dtype != torch.float16 or k_scales.dtype != torch.float16 or \
            q_scales.numel() != heads * ((m - 1) // _Q_ROWS + 1) or k_scales.numel() != heads * ((n - 1) // _K_ROWS + 1):
        raise ValueError("q_scales / k_scales must be fp16 [heads, ceil(M/128)] / [heads, ceil(N/64)]")
    words = torch.empty(heads * tilemix_routing_word_count(m, n, key_tiles_per_group), dtype=torch.int64,
                        device=q_scales.device)
    check(tilemix_routing_policy(q_scales.contiguous(), k_scales.contiguous(), words, heads, m, n,
                                 key_tiles_per_group, max_scale_product, torch.cuda.current_stream(q_scales.device)),
          "tilemix::routing_policy")
    return words


@routing_policy.register_fake
def _(q_scales, k_scales, m, n, key_tiles_per_group, max_scale_product):
    heads = q_scales.shape[0] if q_scales.dim() == 2 else 1
    q16, k32 = (m + 15) // 16, (n + 31) // 32
    groups = (k32 + key_tiles_per_group - 1) // key_tiles_per_group
    return q_scales.new_empty((heads * q16 * ((groups + 63) // 64),), dtype=torch.int64)


@torch.library.custom_op("tilemix::attention_backward", mutates_args=())
def attention_backward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, o: torch.Tensor, do: torch.Tensor,
                       lse: torch.Tensor | None, score_scale: float,
                       causal: bool) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Gradients (dq, dk, dv), fp32 of q's / k's / v's shapes, of the unrouted
    attention o = softmax(score_scale * q k^T [causal]) v, from fp16 q, k, v,
    the fp32 forward output o, the output gradient do (fp16) and, when given,
    the forward's row log-sum-exp lse ([heads, M] fp32 from
    ``attention_lse``; without it the backward recomputes it)."""
    heads, m, n, d = validate_attention_args(q, k, v)
    _require(o.shape == q.shape and o.dtype == torch.float32 and o.device == q.device,
             "o must be a float32 tensor of q's shape on q's device")
    _require(do.shape == q.shape and do.dtype == torch.float16 and do.device == q.device,
             "do must be a float16 tensor of q's shape on q's device")
    if lse is not None:
        _require(lse.numel() == heads * m and lse.dtype == torch.float32 and lse.device == q.device,
                 "lse must be a float32 tensor of heads * M elements on q's device")
    q3, k3, v3 = _heads3(q).contiguous(), _heads3(k).contiguous(), _heads3(v).contiguous()
    o3, do3 = _heads3(o).contiguous(), _heads3(do).contiguous()
    dq = torch.empty(q.shape, dtype=torch.float32, device=q.device)
    dk = torch.empty(k.shape, dtype=torch.float32, device=q.device)
    dv = torch.empty(v.shape, dtype=torch.float32, device=q.device)
    stats = torch.empty((2, heads, m), dtype=torch.float32, device=q.device)
    lse_buf = stats[0] if lse is None else lse.contiguous()
    check(tilemix_attention_backward(q3, k3, v3, o3, do3, dq, dk, dv, lse_buf, stats[1], heads, m, n, d,
                                     score_scale, causal, torch.cuda.current_stream(q.device),
                                     lse_from_forward=lse is not None),
          "tilemix::attention_backward")
    return dq, dk, dv


@attention_backward.register_fake
def _(q, k, v, o, do, lse, score_scale, causal):
    return (q.new_empty(q.shape, dtype=torch.float32), k.new_empty(k.shape, dtype=torch.float32),
            v.new_empty(v.shape, dtype=torch.float32))


@torch.library.custom_op("tilemix::attention_lse", mutates_args=())
def attention_lse(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, score_scale: float,
                  causal: bool) -> tuple[torch.Tensor, torch.Tensor]:
    """Unrouted attention for training: (o fp32 of q's shape, lse fp32
    [heads, M], each row's base-2 log-sum-exp). Its autograd formula runs the
    backward on the saved lse (no recomputation of the row statistics)."""
    heads, m, n, d = validate_attention_args(q, k, v)
    q3, k3, v3 = _heads3(q).contiguous(), _heads3(k).contiguous(), _heads3(v).contiguous()
    out = torch.empty(q.shape, dtype=torch.float32, device=q.device)
    lse = torch.empty((heads, m), dtype=torch.float32, device=q.device)
    check(tilemix_attention_batched_lse(q3, k3, v3, out, lse, heads, m, n, d, score_scale, causal,
                                        torch.cuda.current_stream(q.device)), "tilemix::attention_lse")
    return out, lse


@attention_lse.register_fake
def _(q, k, v, score_scale, causal):
    heads = 1 if q.dim() == 2 else q.shape[0]
    return q.new_empty(q.shape, dtype=torch.float32), q.new_empty((heads, q.shape[-2]), dtype=torch.float32)


def _attention_lse_setup_context(ctx, inputs, output):
    q, k, v, score_scale, causal = inputs
    ctx.set_materialize_grads(False)   # an unused lse gets no gradient tensor
    ctx.score_scale = score_scale
    ctx.causal = causal
    ctx.save_for_backward(q, k, v, *output)


def _attention_lse_backward(ctx, grad, grad_lse):
    if grad_lse is not None:
        raise NotImplementedError("tilemix::attention_lse has no gradient with respect to lse")
    if grad is None:
        return None, None, None, None, None
    q, k, v, o, lse = ctx.saved_tensors
    dq, dk, dv = attention_backward(q, k, v, o, grad.to(torch.float16), lse, ctx.score_scale, ctx.causal)
    return dq.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype), None, None


attention_lse.register_autograd(_attention_lse_backward, setup_context=_attention_lse_setup_context)


def _attention_setup_context(ctx, inputs, output):
    q, k, v, q8, k8, q_scales, k_scales, words, key_tiles_per_group, score_scale, causal = inputs
    ctx.routed = words is not None
    ctx.score_scale = score_scale
    ctx.causal = causal
    ctx.save_for_backward(q, k, v, output)


def _attention_backward(ctx, grad):
    if ctx.routed:
        raise NotImplementedError("tilemix::attention has a gradient for the unrouted (all-FP16) call only")
    q, k, v, o = ctx.saved_tensors
    dq, dk, dv = attention_backward(q, k, v, o, grad.to(torch.float16), None, ctx.score_scale, ctx.causal)
    return dq.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype), None, None, None, None, None, None, None, None


attention.register_autograd(_attention_backward, setup_context=_attention_setup_context)


def tilemix_attention(q, k, v, words=None, *, key_tiles_per_group: int = 2, score_scale: float | None = None,
                      causal: bool = False) -> torch.Tensor:
    """Quantize (when routed) and attend: the whole TileMix hot path as two operators."""
    d = q.shape[-1]
    scale = 1.0 / math.sqrt(d) if score_scale is None else float(score_scale)
    if words is None:
        return attention(q, k, v, None, None, None, None, None, key_tiles_per_group, scale, causal)
    q8, k8, qs, ks = quantize_qk(q, k)
    return attention(q, k, v, q8, k8, qs, ks, words, key_tiles_per_group, scale, causal)
