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
