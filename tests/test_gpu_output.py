"""GPU: strided fp32 / fp16 / bf16 outputs (tilemix_attention_batched_out).

Every element written is exactly the round-to-nearest-even of the fp32 output
the default entry point (tilemix_attention_batched) writes for the same
inputs, in BSHD and padded layouts, on the 16-byte store path and the scalar
one (odd d, odd strides, an unaligned base), and nothing outside the layout's
elements is touched. The fp16 / bf16 outputs are also checked directly
against the fp64 oracle."""
import math

import pytest
import torch

import tilemix_b200 as tm
from tilemix_b200 import workloads

pytestmark = pytest.mark.gpu
SENTINEL = -7.25


def default_output(w, causal, routed, batch, heads_per_batch):
    q, k, v = (w[n].cuda() for n in ("q", "k", "v"))
    kw = {}
    if routed:
        q8, k8, qs, ks = tm.quantize(q, k)
        kw = dict(q8=q8, k8=k8, q_scales=qs, k_scales=ks, words=w["words"].cuda(), key_tiles_per_group=2)
    out = tm.attention(q, k, v, causal=causal, **kw)
    return out, (q, k, v, kw)


def run_out(w, causal, dev_inputs, layout: tm.TileMixOutput):
    q, k, v, kw = dev_inputs
    heads, S, D = w["heads"], w["S"], w["D"]
    routing = quantized = None
    if kw:
        routing = tm.TileMixRouting(kw["words"], kw["words"].numel(), 2)
        quantized = tm.TileMixQuantized(kw["q8"], kw["k8"], kw["q_scales"], kw["k_scales"])
    err = tm.tilemix_attention_batched_out(q, k, v, layout, heads, S, S, D, w["score_scale"], causal, None,
                                           routing, quantized)
    assert err == 0, err
    torch.cuda.synchronize()


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("name,B,H,S,D,causal,routed", [
    ("c3", 2, 3, 300, 128, True, True),
    ("c2", 1, 4, 256, 64, False, True),
    ("c2", 2, 2, 200, 72, False, False),
])
def test_bshd_matches_default_rounded(dtype, name, B, H, S, D, causal, routed):
    w = workloads.make_inputs(name, batch=B, heads=H, seq=S)
    if w["D"] != D:       # shrink / widen the head dim: keep the generator's values, slice or pad
        w = dict(w)
        for n in ("q", "k", "v"):
            t = w[n]
            w[n] = t[..., :D].contiguous() if D <= t.shape[-1] else torch.nn.functional.pad(t, (0, D - t.shape[-1]))
        w["D"] = D
        w["score_scale"] = 1.0 / math.sqrt(D)
    ref, dev_inputs = default_output(w, causal, routed, B, H)
    expect = ref.view(B, H, S, D).permute(0, 2, 1, 3).to(dtype)          # [B, S, H, D]
    out = torch.full((B, S, H, D), SENTINEL, dtype=dtype, device="cuda")
    run_out(w, causal, dev_inputs, tm.TileMixOutput.bshd(out, H))
    assert torch.equal(out, expect)
    err, status = tm.read_and_clear_status()
    assert err == 0 and status == 0


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_padded_and_unaligned_layouts(dtype):
    """Row stride with padding, an odd head stride and a base one element past
    a 16-byte boundary: the scalar store path; padding keeps its sentinel."""
    B, H, S, D = 1, 3, 260, 128
    w = workloads.make_inputs("c3", batch=B, heads=H, seq=S)
    ref, dev_inputs = default_output(w, True, True, B, H)
    row = H * D + 5                      # padded row stride (odd: no 16-byte stores)
    buf = torch.full((1 + S * row,), SENTINEL, dtype=dtype, device="cuda")
    view = buf[1:].view(S, row)          # base one element off alignment
    layout = tm.TileMixOutput(buf[1:], {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}[dtype],
                              H, S * row, D, row)
    run_out(w, True, dev_inputs, layout)
    got = view[:, :H * D].view(S, H, D)
    assert torch.equal(got, ref.view(H, S, D).permute(1, 0, 2).to(dtype))
    assert (view[:, H * D:] == SENTINEL).all() and buf[0].item() == SENTINEL


def test_bhsd_strides_equal_default_layout():
    """heads_per_batch = 1 with the default [heads, S, D] strides reproduces the
    fp32 entry point bit for bit."""
    w = workloads.make_inputs("c5", batch=1, heads=4, seq=384)
    ref, dev_inputs = default_output(w, True, True, 1, 4)
    H, S, D = 4, 384, 128
    out = torch.full((H, S, D), SENTINEL, dtype=torch.float32, device="cuda")
    run_out(w, True, dev_inputs, tm.TileMixOutput(out, 0, 1, S * D, 0, D))
    assert torch.equal(out, ref)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_bshd_against_oracle(dtype):
    """The fp16 / bf16 BSHD output checked directly against the fp64 oracle
    (not only through the fp32 entry point): every element within the parity
    bar plus half an ulp of the output type at the expected value (the
    rounding that storing in that type adds), and the relative L2 error within
    its bar plus the type's unit roundoff."""
    import numpy as np
    import oracle
    B, H, S, D = 2, 2, 300, 128
    w = workloads.make_inputs("c3", batch=B, heads=H, seq=S)
    ref, dev_inputs = default_output(w, True, True, B, H)
    out = torch.full((B, S, H, D), SENTINEL, dtype=dtype, device="cuda")
    run_out(w, True, dev_inputs, tm.TileMixOutput.bshd(out, H))
    heads = B * H
    q, k, v = (w[n].numpy() for n in ("q", "k", "v"))
    q8, qs = oracle.quantize(q, 128)
    k8, ks = oracle.quantize(k, 64)
    words = w["words"].numpy()
    wc = words.size // heads
    bits = np.stack([oracle.decode_routing(words[h * wc:(h + 1) * wc], S, S, 2) for h in range(heads)])
    expect = oracle.tilemix_attention(q, k, v, q8, k8, qs, ks, bits, w["score_scale"], causal=True)
    got = out.float().cpu().permute(0, 2, 1, 3).reshape(heads, S, D).numpy().astype(np.float64)
    unit = {torch.float16: 2.0 ** -11, torch.bfloat16: 2.0 ** -8}[dtype]
    bound = 2e-3 + unit * np.abs(expect) + 2.0 ** -24      # the last term covers fp16 subnormals
    assert np.all(np.abs(got - expect) <= bound), float(np.max(np.abs(got - expect) - bound))
    rel_l2 = float(np.linalg.norm(got - expect) / np.linalg.norm(expect))
    assert rel_l2 <= 1e-3 + unit, rel_l2
    err, status = tm.read_and_clear_status()
    assert err == 0 and status == 0
