"""The reference test suite's cases and input patterns, restated for our tests.

Follows the reference's src/tests/tilemix_test.cu: the deterministic mt19937
input generator (:43-54, implemented in oracle/tilemix_oracle.c), the pattern
overrides (:55-134), the quantizer cases (:364-382), the routing-mask builder
(:424-448) and the case lists (:554-576, :592-605). Test infrastructure only.
"""
from __future__ import annotations

import numpy as np

import oracle

H = np.float16

# tilemix_test.cu:592-605 -- dense FP64-reference cases (M, N, d, pattern, default_stream)
DENSE_D_SWEEP = [1, 15, 16, 17, 31, 32, 33, 49, 63, 64, 65, 81, 97, 113, 127, 128]
DENSE_CASES = [(3, 33, d, "random", False) for d in DENSE_D_SWEEP] + [
    (1, 1, 1, "random", False), (3, 5, 7, "random", False),
    (15, 31, 15, "random", False), (16, 32, 16, "random", False), (17, 33, 17, "random", False),
    (31, 63, 31, "random", False), (32, 64, 32, "random", False), (33, 65, 33, "random", False),
    (35, 67, 65, "random", False), (17, 65, 128, "random", False),
    (17, 1, 128, "random", False), (17, 33, 17, "random", True),
    (17, 65, 1, "rising", False), (17, 65, 1, "falling", False), (17, 129, 1, "alternating", False),
    (17, 65, 1, "late-extreme", False), (17, 33, 1, "negative", False),
    (17, 33, 17, "zeros", False), (17, 33, 17, "uniform", False), (17, 33, 17, "zero-v", False),
    (17, 65, 17, "constant-v", False), (2, 32, 17, "cancellation", False),
    (17, 33, 1, "large-dot", False),
    (3, 2051, 17, "random", False), (1, 4097, 128, "uniform", False),
]

# tilemix_test.cu:366-368 -- quantizer exact-bytes cases (M, N, d, pattern)
QUANT_CASES = [(129, 65, 17, "zeros"), (129, 65, 1, "rounding"), (129, 65, 3, "tiny"),
               (3, 5, 128, "max-range"), (137, 73, 31, "random"), (129, 131, 17, "block-outliers")]
ROUNDING_TIES = [127.0, -127.0, 0.5, -0.5, 1.5, -1.5, 126.5, -126.5]
ROUNDING_KNOWN = [127, -127, 1, -1, 2, -2, 127, -127]

# tilemix_test.cu:554-576 -- routing cases ((M, N, d, pattern, default_stream), group)
INT_MAX = 2**31 - 1
ROUTING_SHAPES = [
    ((35, 67, 17, "random", False), 2), ((17, 2048, 5, "random", False), 1),
    ((17, 2049, 5, "random", False), 1), ((17, 4099, 5, "random", False), 2),
    ((35, 163, 17, "random", False), 3), ((17, 65, 17, "random", False), INT_MAX),
    ((17, 4097, 3, "random", False), 1), ((129, 131, 17, "block-outliers", True), 1),
    ((17, 65, 17, "zeros", False), 2), ((17, 65, 1, "rising", False), 1),
    ((17, 65, 1, "falling", False), 1), ((17, 129, 1, "alternating", False), 1),
    ((17, 65, 1, "late-extreme", False), 1), ((17, 33, 128, "max-int8", False), 1),
]
ROUTING_PATTERNS = ["fp16", "int8-requested", "mixed"]
ROUTING_D_SWEEP = [1, 15, 16, 17, 31, 32, 33, 63, 64, 65, 127, 128]


def routing_cases():
    """(shape, group, pattern, trace) in the reference's order."""
    out = []
    for shape, group in ROUTING_SHAPES:
        for pattern in ROUTING_PATTERNS:
            out.append((shape, group, pattern, True))
    for d in ROUTING_D_SWEEP:
        for pattern in ROUTING_PATTERNS:
            out.append(((3, 33, d, "random", False), 1, pattern, True))
    out.append(((17, 2051, 5, "random", False), 1, "implicit-fp16", True))
    out.append(((35, 67, 17, "random", False), 2, "mixed", False))
    return out


def inputs(m: int, n: int, d: int, pattern: str):
    """Q, K, V fp16 arrays for a reference test pattern (tilemix_test.cu:43-134)."""
    q, k, v = (a.copy() for a in oracle.reference_inputs(m, n, d))
    if pattern == "zeros":
        q[:] = 0; k[:] = 0; v[:] = 0
        return q, k, v
    if pattern == "random":
        return q, k, v
    if pattern == "block-outliers":
        assert m >= 129 and n >= 129
        q[127, 0] = 8.0; q[128, 0] = 0.125
        k[63, 0] = -16.0; k[128, 0] = 0.25
        return q, k, v
    if pattern == "max-int8":
        q[:] = 1.0; k[:] = 1.0; k[0, :] = -1.0
        return q, k, v
    if pattern == "zero-v":
        v[:] = 0
        return q, k, v
    if pattern == "constant-v":
        v[:] = ((np.arange(d) % 7 - 3) * 0.25).astype(H)[None, :]
        return q, k, v
    if pattern == "cancellation":
        q[:] = 0
        v[:] = np.where(np.arange(n) % 2 == 1, -1.0, 1.0).astype(H)[:, None]
        return q, k, v
    if pattern == "large-dot":
        q[:] = 1000.0; k[:] = -1000.0; k[0, :] = 1000.0
        return q, k, v
    q[:] = 0
    if pattern == "uniform":
        return q, k, v
    k[:] = 0
    q[:, 0] = 1.0
    for key in range(n):
        tile = key // 32
        if pattern == "rising":
            score = 4.0 * (tile - 1)
            value = 1.0 if tile == 0 else (-1.0 if tile == 1 else 2.0)
        elif pattern == "falling":
            score = 4.0 * (1 - tile)
            value = 1.0 if tile == 0 else (-1.0 if tile == 1 else 2.0)
        elif pattern == "alternating":
            assert tile < 5
            score = [0, 4, -2, 8, 10][tile]
            value = [1, -1, 2, -2, 3][tile]
        elif pattern == "late-extreme":
            score = 1000.0 if key == n - 1 else 0.0
            value = 3.0 if key == n - 1 else 1.0
        elif pattern == "negative":
            score = -1000.0
            value = (key % 7 - 3) * 0.25
        else:
            raise ValueError(pattern)
        k[key, 0] = score
        v[key, :] = value
    return q, k, v


def quant_inputs(m: int, n: int, d: int, pattern: str):
    """Q, K for a quantizer case (tilemix_test.cu:370-382)."""
    q, k, _ = inputs(m, n, d, "block-outliers" if pattern == "block-outliers" else "random")
    for a in (q, k):
        flat = a.reshape(-1)
        idx = np.arange(flat.size)
        if pattern == "zeros":
            flat[:] = 0
        elif pattern == "rounding":
            flat[:] = np.array(ROUNDING_TIES, np.float32)[idx % 8].astype(H)
        elif pattern == "tiny":
            flat[:] = np.where(idx % 2 == 1, -(2.0**-24), 2.0**-24).astype(H)
        elif pattern == "max-range":
            flat[:] = np.where(idx % 2 == 1, -65504.0, 65504.0).astype(H)
    return q, k


def routing_words(m: int, n: int, group: int, pattern: str):
    """Mask words and expected per-(query tile, key tile) bits (tilemix_test.cu:425-448).
    Words start all-ones, so bits past the last group stay set, as in the reference."""
    query_tiles = (m + 15) // 16
    key_tiles = (n + 31) // 32
    groups = (key_tiles + group - 1) // group
    wpr = (groups + 63) // 64
    words = np.full(query_tiles * wpr, np.uint64(0xFFFFFFFFFFFFFFFF), np.uint64)
    bits = np.zeros((query_tiles, key_tiles), np.uint8)
    for row in range(query_tiles):
        tile = 0
        for g in range(groups):
            bit = pattern == "int8-requested" or (pattern == "mixed" and (g + row + g // 64) % 2 == 0)
            flag = np.uint64(1) << np.uint64(g % 64)
            if bit:
                words[row * wpr + g // 64] |= flag
            else:
                words[row * wpr + g // 64] &= ~flag
            for _ in range(group):
                if tile >= key_tiles:
                    break
                bits[row, tile] = bit
                tile += 1
    return words, bits


def closed_form(pattern: str, v: np.ndarray, n: int) -> float:
    """Closed-form softmax expectations of the analytic patterns (tilemix_test.cu:243-258)."""
    e = np.exp
    if pattern == "rising":
        a, b = 32 * e(-8.0), 32 * e(-4.0)
        return (a - b + 2) / (a + b + 1)
    if pattern == "falling":
        b, c = 32 * e(-4.0), e(-8.0)
        return (32 - b + 2 * c) / (32 + b + c)
    if pattern == "alternating":
        a, b, c, x = 32 * e(-10.0), 32 * e(-6.0), 32 * e(-12.0), 32 * e(-2.0)
        return (a - b + 2 * c - 2 * x + 3) / (a + b + c + x + 1)
    if pattern == "late-extreme":
        return 3.0
    if pattern == "negative":
        return float(v.astype(np.float64).sum() / n)
    raise ValueError(pattern)


def compare_stats(actual: np.ndarray, expected: np.ndarray):
    """(max_abs, rel_l2) of actual vs expected in float64."""
    a = np.asarray(actual, np.float64)
    e = np.asarray(expected, np.float64)
    err = a - e
    max_abs = float(np.abs(err).max()) if err.size else 0.0
    denom = float(np.linalg.norm(e))
    rel_l2 = float(np.linalg.norm(err) / denom) if denom > 0 else float(np.linalg.norm(err))
    return max_abs, rel_l2


# Parity tolerance of the north star: max-abs 2e-3 and relative-L2 1e-3 (fp32 output
# vs the reference's fp64 mixed-precision emulation).
MAX_ABS_TOL = 2e-3
REL_L2_TOL = 1e-3
