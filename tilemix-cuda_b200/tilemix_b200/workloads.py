"""Seeded synthetic workloads for the five BASELINE configurations.

The reference measures on no public dataset; its configs describe synthetic
inputs, generated here on the host with torch's CPU generator:
  Q, K, V = randn(B, H, S, D) * sigma  (drawn in that order), optional outlier
  channels (ceil(1% of D) picked by randperm(D) from the same generator, x20 in
  Q, K and V before the fp16 cast), then an INT8 block mask
  rand(B, H, ceil(S/64), ceil(S/64)) < p over 64x64 tiles (config 5 forces the
  diagonal band kb in {qb-1, qb} to FP16). Layout is contiguous [B*H, S, D], so
  each head is the reference's 2-D [S, D] layout. The 64x64 mask is packed into
  the reference's routing words with key_tiles_per_group = 2, each 64-row mask
  row replicated into its four 16-row query tiles.
"""
from __future__ import annotations

import math

import numpy as np
import torch

CONFIGS = {
    "c1": dict(B=1, H=1, S=256, D=64, causal=False, seed=0, p=0.5, sigma=1.0, outliers=False, band=False),
    "c2": dict(B=4, H=16, S=1024, D=64, causal=False, seed=1, p=0.5, sigma=1.0, outliers=False, band=False),
    "c3": dict(B=8, H=32, S=4096, D=128, causal=True, seed=2, p=0.75, sigma=1.0, outliers=True, band=False),
    "c4": dict(B=1, H=32, S=32768, D=128, causal=False, seed=3, p=0.5, sigma=1.0, outliers=False, band=False),
    "c5": dict(B=16, H=32, S=2048, D=128, causal=True, seed=4, p=0.5, sigma=0.5, outliers=False, band=True),
}

P_F16_PUBLISHED = 2.25e15   # NVIDIA B200 dense FP16/BF16 tensor peak, FLOP/s
P_I8_PUBLISHED = 4.5e15     # NVIDIA B200 dense INT8 tensor peak, OP/s


def config(name: str, **overrides) -> dict:
    cfg = dict(CONFIGS[name])
    cfg.update({k: v for k, v in overrides.items() if v is not None})
    cfg["name"] = name
    return cfg


def pack_block_mask64(block_mask: np.ndarray, S_q: int, S_k: int) -> np.ndarray:
    """[heads, ceil(S_q/64), ceil(S_k/64)] 0/1 -> routing words [heads * word_count]
    with key_tiles_per_group = 2 (one 64-key group per mask column)."""
    heads = block_mask.shape[0]
    q_tiles = (S_q + 15) // 16
    key_tiles = (S_k + 31) // 32
    groups = (key_tiles + 1) // 2
    wpr = (groups + 63) // 64
    rows = np.repeat(block_mask.astype(np.uint64), 4, axis=1)[:, :q_tiles, :groups]
    padded = np.zeros((heads, q_tiles, wpr * 64), np.uint64)
    padded[:, :, :groups] = rows
    shifts = np.arange(64, dtype=np.uint64)
    words = (padded.reshape(heads, q_tiles, wpr, 64) << shifts).sum(axis=-1, dtype=np.uint64)
    return np.ascontiguousarray(words.reshape(-1))


def make_inputs(name: str, p: float | None = None, batch: int | None = None,
                heads: int | None = None, seq: int | None = None, seed: int | None = None,
                device: str = "cpu") -> dict:
    """Tensors for a config. Returns q, k, v fp16 [B*H, S, D], the 64x64 block
    mask [B*H, S/64, S/64] uint8, routing words (host), score scale and the
    config dict. Overrides shrink a config for tests (same generator order).
    device="cuda" draws with a CUDA generator instead (same distributions,
    different numbers; used by the benchmark to avoid minutes of host RNG)."""
    cfg = config(name, p=p, B=batch, H=heads, S=seq, seed=seed)
    B, H, S, D = cfg["B"], cfg["H"], cfg["S"], cfg["D"]
    g = torch.Generator(device=device).manual_seed(cfg["seed"])
    q = torch.randn((B, H, S, D), generator=g, device=device) * cfg["sigma"]
    k = torch.randn((B, H, S, D), generator=g, device=device) * cfg["sigma"]
    v = torch.randn((B, H, S, D), generator=g, device=device) * cfg["sigma"]
    if cfg["outliers"]:
        n_out = math.ceil(0.01 * D)
        channels = torch.randperm(D, generator=g, device=device)[:n_out]
        for t in (q, k, v):
            t[..., channels] *= 20.0
    qb = (S + 63) // 64
    mask = (torch.rand((B, H, qb, qb), generator=g, device=device) < cfg["p"]).to(torch.uint8)
    if cfg["band"]:
        idx = torch.arange(qb, device=device)
        band = (idx[None, :] == idx[:, None]) | (idx[None, :] == idx[:, None] - 1)
        mask[..., band] = 0
    q16, k16, v16 = (t.to(torch.float16).reshape(B * H, S, D).contiguous() for t in (q, k, v))
    del q, k, v
    mask = mask.reshape(B * H, qb, qb).contiguous().cpu()
    words = torch.from_numpy(pack_block_mask64(mask.numpy(), S, S))
    return dict(q=q16, k=k16, v=v16, mask=mask, words=words, score_scale=1.0 / math.sqrt(D),
                cfg=cfg, heads=B * H, S=S, D=D)


def realised_int8_fraction(mask: torch.Tensor | np.ndarray, causal: bool) -> float:
    """INT8 fraction over the unmasked 64x64 blocks (causal: kb <= qb)."""
    m = mask.numpy() if isinstance(mask, torch.Tensor) else mask
    qb = m.shape[-1]
    if causal:
        keep = np.tril(np.ones((qb, qb), bool))
        return float(m[:, keep].mean())
    return float(m.mean())


def int8_fraction_from_words(words: np.ndarray, heads: int, S: int, causal: bool,
                             key_tiles_per_group: int = 2) -> float:
    """INT8 share of the QK work a set of routing words selects: over the
    (16-row query tile, 32-key tile) pairs the kernel computes (causal: key
    tiles that start at or before the tile's last row)."""
    q16, k32 = (S + 15) // 16, (S + 31) // 32
    groups = (k32 + key_tiles_per_group - 1) // key_tiles_per_group
    wpr = (groups + 63) // 64
    w = np.ascontiguousarray(words, dtype=np.uint64).reshape(heads, q16, wpr)
    bits = np.unpackbits(w.view(np.uint8), axis=-1, bitorder="little").reshape(heads, q16, wpr * 64)
    tile_bits = np.repeat(bits[:, :, :groups], key_tiles_per_group, axis=-1)[:, :, :k32]
    if causal:
        keep = (np.arange(k32)[None, :] * 32) <= (np.arange(q16)[:, None] * 16 + 15)
        return float(tile_bits[:, keep].mean())
    return float(tile_bits.mean())


def effective_flops(cfg: dict, heads: int | None = None) -> float:
    """F_eff = 4 * B*H * S^2 * D, halved for causal (flash-attention convention)."""
    bh = heads if heads is not None else cfg["B"] * cfg["H"]
    f = 4.0 * bh * cfg["S"] ** 2 * cfg["D"]
    return f * (0.5 if cfg["causal"] else 1.0)


def mix_peak(f_eff: float, f_real: float, p_f16: float = P_F16_PUBLISHED,
             p_i8: float = P_I8_PUBLISHED) -> float:
    """P_mix = F_eff / (F_QK,i8/P_i8 + (F_QK,f16 + F_PV)/P_f16), F_QK = F_PV = F_eff/2."""
    f_qk = f_pv = f_eff / 2
    f_i8 = f_real * f_qk
    return f_eff / (f_i8 / p_i8 + (f_qk - f_i8 + f_pv) / p_f16)
