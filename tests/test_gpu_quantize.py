"""GPU: stage-1 quantizer, bit-exact against the oracle and the reference's
golden bytes (tilemix_test.cu:364-422), including guards, immutability, the
scalar (unaligned / odd-d) path and BASELINE-sized batches."""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
import refcases
from gpu_util import dev, guarded, host, quantize_gpu, I8_GUARD, SCALE_GUARD
import tilemix_b200 as tm

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden" / "reference_golden.npz"


def test_reference_quantizer_cases_bit_exact():
    g = np.load(GOLDEN)
    index = json.loads(bytes(g["index"]).decode())
    stream = torch.cuda.Stream()
    for i, (m, n, d, pattern) in enumerate(index["quant"]):
        q, k = refcases.quant_inputs(m, n, d, pattern)
        q8, k8, qs, ks = quantize_gpu(q, k, stream=stream)
        assert np.array_equal(q8, g[f"quant{i}_q8"]), pattern
        assert np.array_equal(k8, g[f"quant{i}_k8"]), pattern
        assert np.array_equal(qs.view(np.uint16), g[f"quant{i}_qs"]), pattern
        assert np.array_equal(ks.view(np.uint16), g[f"quant{i}_ks"]), pattern
        if pattern == "rounding":
            assert q8.reshape(-1)[:8].tolist() == refcases.ROUNDING_KNOWN


@pytest.mark.parametrize("m,n,d", [(1, 1, 1), (128, 64, 128), (129, 65, 8), (300, 1000, 64),
                                   (1000, 1003, 128), (257, 200, 96), (77, 93, 13)])
def test_random_shapes_bit_exact(m, n, d):
    rng = np.random.default_rng(m * 7 + n + d)
    q = (rng.standard_normal((m, d)) * rng.uniform(0.01, 50)).astype(np.float16)
    k = (rng.standard_normal((n, d)) * rng.uniform(0.01, 50)).astype(np.float16)
    q8, k8, qs, ks = quantize_gpu(q, k)
    eq8, eqs = oracle.quantize(q, 128)
    ek8, eks = oracle.quantize(k, 64)
    assert np.array_equal(q8, eq8) and np.array_equal(k8, ek8)
    assert np.array_equal(qs.view(np.uint16), eqs.view(np.uint16))
    assert np.array_equal(ks.view(np.uint16), eks.view(np.uint16))


def test_unaligned_pointers_take_scalar_path_bit_exact():
    """Outputs offset by one element (as the reference's guard layout does) and
    inputs offset by one half are not vector-aligned."""
    rng = np.random.default_rng(3)
    m, n, d = 300, 260, 64
    q = rng.standard_normal((m, d)).astype(np.float16)
    k = rng.standard_normal((n, d)).astype(np.float16)
    qd = dev(np.concatenate([[0], q.reshape(-1)]).astype(np.float16))
    kd = dev(np.concatenate([[0], k.reshape(-1)]).astype(np.float16))
    q8 = guarded(q.size, torch.int8, I8_GUARD)
    k8 = guarded(k.size, torch.int8, I8_GUARD)
    qs = guarded(3, torch.float16, SCALE_GUARD)
    ks = guarded(5, torch.float16, SCALE_GUARD)
    assert tm.quantize_tilemix_qk(qd.data_ptr() + 2, kd.data_ptr() + 2, q8[1:], k8[1:], qs[1:], ks[1:],
                                  m, n, d) == 0
    torch.cuda.synchronize()
    eq8, eqs = oracle.quantize(q, 128)
    ek8, eks = oracle.quantize(k, 64)
    assert np.array_equal(host(q8)[1:-1].reshape(m, d), eq8)
    assert np.array_equal(host(k8)[1:-1].reshape(n, d), ek8)
    assert np.array_equal(host(qs)[1:-1].view(np.uint16), eqs.view(np.uint16))
    assert np.array_equal(host(ks)[1:-1].view(np.uint16), eks.view(np.uint16))
    assert host(q8)[0] == I8_GUARD and host(k8)[-1] == I8_GUARD


@pytest.mark.parametrize("name", ["c3", "c5"])
def test_baseline_batch_bit_exact(name):
    """Full-width heads of the BASELINE configs (with config 3's x20 outlier channels)."""
    from tilemix_b200 import workloads
    w = workloads.make_inputs(name, batch=1, heads=4)
    q, k = w["q"].numpy(), w["k"].numpy()
    q8, k8, qs, ks = quantize_gpu(q, k, heads=w["heads"])
    eq8, eqs = oracle.quantize(q, 128)
    ek8, eks = oracle.quantize(k, 64)
    assert np.array_equal(q8, eq8) and np.array_equal(k8, ek8)
    assert np.array_equal(qs.view(np.uint16), eqs.view(np.uint16).reshape(qs.shape))
    assert np.array_equal(ks.view(np.uint16), eks.view(np.uint16).reshape(ks.shape))


def _all_fp16_up_to(absmax: float) -> np.ndarray:
    """Every finite fp16 value v with |v| <= absmax (both signs, with zero)."""
    bits = np.arange(0, 0x7C00, dtype=np.uint16)
    pos = bits.view(np.float16)
    pos = pos[pos.astype(np.float32) <= np.float32(absmax)]
    return np.concatenate([pos, -pos[1:]])


@pytest.mark.parametrize("absmax", [1.0, 127.0, 3.140625, 100.0, 65504.0, 2.0 ** -10, 6.0e-8])
def test_exhaustive_fp16_values_bit_exact(absmax):
    """Every fp16 value within one block's absmax, so every tie (x / scale exactly
    k + 1/2) and near-tie of the half-away-from-zero rounding is exercised on the
    quantizer's vector path, for Q (128-row) and K (64-row) blocks."""
    vals = _all_fp16_up_to(absmax)
    d = 128
    per_block = 64 * d - 1                      # one slot per block holds the absmax
    nblocks = -(-vals.size // per_block)
    rows = []
    for b in range(nblocks):
        chunk = vals[b * per_block:(b + 1) * per_block]
        block = np.zeros(64 * d, np.float16)
        block[0] = np.float16(absmax)
        block[1:1 + chunk.size] = chunk
        rows.append(block.reshape(64, d))
    x = np.concatenate(rows)                     # 64-row K blocks; Q blocks pair them
    if x.shape[0] % 128:
        x = np.concatenate([x, np.zeros((64, d), np.float16)])
    q8, k8, qs, ks = quantize_gpu(x, x)
    eq8, eqs = oracle.quantize(x, 128)
    ek8, eks = oracle.quantize(x, 64)
    assert np.array_equal(q8, eq8) and np.array_equal(k8, ek8)
    assert np.array_equal(qs.view(np.uint16), eqs.view(np.uint16))
    assert np.array_equal(ks.view(np.uint16), eks.view(np.uint16))


def test_nan_and_inf_blocks_take_the_exact_path():
    """Blocks holding a NaN or an inf leave the branch-free rounding for the
    element-wise exact path (the reference GPU kernel's semantics): a NaN input
    gives 0 and does not enter the absmax; a block whose absmax is inf has an
    inf scale and all-zero bytes. Neighbouring finite blocks are unaffected."""
    rng = np.random.default_rng(9)
    d = 64
    q = rng.standard_normal((512, d)).astype(np.float16)
    q[5, 7] = np.nan                  # Q block 0 (and K block 0)
    q[300, 1] = -np.inf               # Q block 2 (and K block 4)
    q8, k8, qs, ks = quantize_gpu(q, q)
    finite = np.where(np.isnan(q), np.float16(0), q)
    for got8, got_s, rows in ((q8, qs, 128), (k8, ks, 64)):
        for b in range(512 // rows):
            blk = slice(b * rows, (b + 1) * rows)
            if np.isinf(q[blk]).any():
                assert np.isinf(got_s[b]) and not got8[blk].any()
                continue
            e8, es = oracle.quantize(finite[blk], rows)
            e8 = np.where(np.isnan(q[blk]), np.int8(0), e8)
            assert np.array_equal(got8[blk], e8), (rows, b)
            assert got_s[b].view(np.uint16) == es.view(np.uint16)[0], (rows, b)
