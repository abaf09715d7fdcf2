"""GPU test helpers: device buffers with guard sentinels, calls through the C-ABI
(tilemix_b200 -> libtilemix_b200.so), and host copies for oracle comparison."""
from __future__ import annotations

import numpy as np
import torch

import tilemix_b200 as tm

DEV = "cuda:0"
OUT_GUARD = -12345.25          # tilemix_test.cu:273
I8_GUARD = -128                # 0x80, tilemix_test.cu:406
SCALE_GUARD = 60000.0          # tilemix_test.cu:397
BITS_GUARD = 0xA5              # tilemix_test.cu:468
DOT_GUARD = 0x2468ACE          # tilemix_test.cu:476


def dev(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def guarded(count: int, dtype, guard, fill=None) -> torch.Tensor:
    """[count + 2] device buffer: guard, fill..., guard."""
    t = torch.full((count + 2,), guard if fill is None else fill, dtype=dtype, device=DEV)
    t[0] = guard
    t[-1] = guard
    return t


def host(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().numpy()


def quantize_gpu(q: np.ndarray, k: np.ndarray, stream=None, heads: int | None = None):
    """Quantize through the C-ABI with guard sentinels; returns host arrays and
    asserts the guards survived."""
    qd, kd = dev(q), dev(k)
    if heads is None:
        m, d = q.shape[-2], q.shape[-1]
        n = k.shape[-2]
        heads = 1 if q.ndim == 2 else q.shape[0]
    else:
        m, d, n = q.shape[-2], q.shape[-1], k.shape[-2]
    qb, kb = (m - 1) // 128 + 1, (n - 1) // 64 + 1
    q8 = guarded(q.size, torch.int8, I8_GUARD)
    k8 = guarded(k.size, torch.int8, I8_GUARD)
    qs = guarded(heads * qb, torch.float16, SCALE_GUARD)
    ks = guarded(heads * kb, torch.float16, SCALE_GUARD)
    if heads == 1 and q.ndim == 2:
        err = tm.quantize_tilemix_qk(qd, kd, q8[1:], k8[1:], qs[1:], ks[1:], m, n, d, stream)
    else:
        err = tm.quantize_tilemix_qk_batched(qd, kd, q8[1:], k8[1:], qs[1:], ks[1:], heads, m, n, d, stream)
    assert err == 0, err
    torch.cuda.synchronize()
    out = [host(t) for t in (q8, k8, qs, ks)]
    for a, g in zip(out, (I8_GUARD, I8_GUARD, SCALE_GUARD, SCALE_GUARD)):
        assert a[0] == g and a[-1] == g, "quantizer guard overwritten"
    assert np.array_equal(host(qd).view(np.uint16), q.view(np.uint16)) and \
        np.array_equal(host(kd).view(np.uint16), k.view(np.uint16)), "quantizer modified its input"
    q8h = out[0][1:-1].reshape(q.shape)
    k8h = out[1][1:-1].reshape(k.shape)
    qsh = out[2][1:-1].reshape(heads, qb)
    ksh = out[3][1:-1].reshape(heads, kb)
    if q.ndim == 2:
        qsh, ksh = qsh[0], ksh[0]
    return q8h, k8h, qsh, ksh
