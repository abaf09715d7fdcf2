"""PyTorch operators over the C-ABI: ``torch.ops.tilemix.quantize_qk``,
``torch.ops.tilemix.attention`` and ``torch.ops.tilemix.attention_bshd``.

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

from . import (TileMixOutput, TileMixQuantized, TileMixRouting, check, quantize_tilemix_qk_batched,
               tilemix_attention_batched, tilemix_attention_batched_out, validate_attention_args,
               validate_quantize_args)

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


def tilemix_attention(q, k, v, words=None, *, key_tiles_per_group: int = 2, score_scale: float | None = None,
                      causal: bool = False) -> torch.Tensor:
    """Quantize (when routed) and attend: the whole TileMix hot path as two operators."""
    d = q.shape[-1]
    scale = 1.0 / math.sqrt(d) if score_scale is None else float(score_scale)
    if words is None:
        return attention(q, k, v, None, None, None, None, None, key_tiles_per_group, scale, causal)
    q8, k8, qs, ks = quantize_qk(q, k)
    return attention(q, k, v, q8, k8, qs, ks, words, key_tiles_per_group, scale, causal)
