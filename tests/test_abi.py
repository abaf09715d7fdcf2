"""CPU: the C-ABI library loads, exports every declared symbol, and enforces the
reference's argument-validation contract without touching a GPU
(reference src/tests/tilemix_test.cu:157-235, the `--cpu-only` checks)."""
import ctypes
import re
import subprocess
from pathlib import Path

import pytest

import tilemix_b200 as tm
from tilemix_b200 import _build

REPO = Path(__file__).resolve().parents[1]
INVALID, NOT_SUPPORTED = tm.cudaErrorInvalidValue, tm.cudaErrorNotSupported


def declared_c_functions():
    names = set()
    for header in sorted((REPO / "include").glob("*.h")):
        text = header.read_text()
        if 'extern "C"' not in text:
            continue
        body = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names.update(re.findall(r"^\s*(?:int|size_t|void|unsigned int|float)\s+(tilemix_\w+)\s*\(", body, re.M))
    return sorted(names)


def test_library_loads_and_exports_every_declared_symbol():
    names = declared_c_functions()
    assert len(names) >= 10
    for name in names:
        assert hasattr(tm.lib, name), name
    assert set(names) == set(tm.C_ABI_SYMBOLS)
    assert tm.lib.tilemix_abi_version() == 1


def test_cpp_dropin_symbols_exported():
    out = subprocess.run(["nm", "-D", "-C", str(tm.LIB_PATH)], capture_output=True, text=True).stdout
    for sig in ("quantize_tilemix_qk(__half const*, __half const*, signed char*, signed char*, __half*, __half*, int, int, int, CUstream_st*)",
                "launch_fused_fp16_attention(__half const*, __half const*, __half const*, float*, int, int, int, float, CUstream_st*, TileMixRouting const&, TileMixQuantized const&)",
                "tilemix_attention_batched(", "quantize_tilemix_qk_batched("):
        assert sig in out, sig


def test_library_is_sm100a_only():
    assert _build.ARCH == ["-gencode", "arch=compute_100a,code=sm_100a"]


def test_layout_constants_match_reference():
    """tilemix_test.cu:186-191 and the routing-word table :208-217."""
    assert [tm.tilemix_shared_bytes(d, False) for d in (1, 17, 128, 129)] == [4608, 7168, 22528, 0]
    assert tm.tilemix_shared_bytes(128, True) == 28672 and tm.tilemix_shared_bytes(17, True) == 8704
    assert (tm.kTileMixQQuantRows, tm.kTileMixKQuantRows) == (128, 64)
    rc = tm.tilemix_routing_word_count
    assert rc(17, 2048, 1) == 2 and rc(17, 2049, 1) == 4 and rc(17, 4097, 2) == 4
    assert rc(17, 4097, 1) == 6 and rc(17, 2**31 - 1, 2**31 - 1) == 2
    assert rc(0, 1, 1) == 0 and rc(1, 0, 1) == 0 and rc(1, 1, 0) == 0
    assert tm.tilemix_b200_shared_bytes(128) <= 227 * 1024
    assert tm.tilemix_b200_shared_bytes(64) > 114 * 1024   # one CTA (one TMEM owner) per SM
    assert tm.tilemix_b200_shared_bytes(129) == 0


def test_argument_validation_without_cuda():
    """Every invalid call returns its error code before any CUDA call."""
    x = ctypes.create_string_buffer(64)
    X = ctypes.addressof(x)
    f = tm.launch_fused_fp16_attention
    assert f(None, X, X, X, 1, 1, 1, 1.0) == INVALID
    assert f(X, None, X, X, 1, 1, 1, 1.0) == INVALID
    assert f(X, X, None, X, 1, 1, 1, 1.0) == INVALID
    assert f(X, X, X, None, 1, 1, 1, 1.0) == INVALID
    for bad in (0, -1):
        assert f(X, X, X, X, bad, 1, 1, 1.0) == INVALID
        assert f(X, X, X, X, 1, bad, 1, 1.0) == INVALID
        assert f(X, X, X, X, 1, 1, bad, 1.0) == INVALID
    for d in (129, 2**31 - 1):
        assert f(X, X, X, X, 1, 1, d, 1.0) == NOT_SUPPORTED
    for s in (float("nan"), float("inf"), float("-inf")):
        assert f(X, X, X, X, 1, 1, 1, s) == INVALID
    q = tm.quantize_tilemix_qk
    assert q(None, X, X, X, X, X, 1, 1, 1) == INVALID
    assert q(X, X, None, X, X, X, 1, 1, 1) == INVALID
    assert q(X, X, X, X, None, X, 1, 1, 1) == INVALID
    assert q(X, X, X, X, X, X, 0, 1, 1) == INVALID
    assert q(X, X, X, X, X, X, 1, 1, 129) == NOT_SUPPORTED
    assert f(X, X, X, X, 1, 1, 1, 1.0, quantized=tm.TileMixQuantized(q=X)) == INVALID
    for group in (0, -1):
        assert f(X, X, X, X, 1, 1, 1, 1.0, routing=tm.TileMixRouting(None, 0, group)) == INVALID
    assert f(X, X, X, X, 1, 1, 1, 1.0, routing=tm.TileMixRouting(X, 1, 1)) == INVALID
    for routing in (tm.TileMixRouting(None, 1, 1), tm.TileMixRouting(X, 0, 1), tm.TileMixRouting(X, 3, 1)):
        assert f(X, X, X, X, 17, 2049, 1, 1.0, routing=routing) == INVALID


def test_batched_validation_without_cuda():
    x = ctypes.create_string_buffer(64)
    X = ctypes.addressof(x)
    b = tm.tilemix_attention_batched
    assert b(X, X, X, X, 0, 4, 4, 16, 1.0) == INVALID
    # 2 heads need 2 x word_count(17, 2049, 1) = 8 words
    quant = tm.TileMixQuantized(X, X, X, X)
    assert b(X, X, X, X, 2, 17, 2049, 16, 1.0, routing=tm.TileMixRouting(X, 7, 1), quantized=quant) == INVALID
    assert tm.quantize_tilemix_qk_batched(X, X, X, X, X, X, 0, 4, 4, 16) == INVALID
    assert tm.quantize_tilemix_qk_batched(X, X, X, X, X, X, 2, 4, 4, 200) == NOT_SUPPORTED


def test_demo_driver_built():
    assert _build.DEMO_BIN.exists()


def test_from_host_validation_without_cuda():
    """The host-buffer pipeline rejects bad arguments before any CUDA call."""
    x = ctypes.create_string_buffer(64)
    X = ctypes.addressof(x)
    full = tm.TileMixDeviceBuffers(X, X, X, X, X, X, X, X, X)
    f = tm.tilemix_attention_from_host
    assert f(None, X, X, X, X, full, 1, 4, 4, 16, 1.0) == INVALID
    assert f(X, X, X, X, None, full, 1, 4, 4, 16, 1.0) == INVALID
    assert f(X, X, X, X, X, None, 1, 4, 4, 16, 1.0) == INVALID
    assert f(X, X, X, X, X, tm.TileMixDeviceBuffers(X, X, X, o=None), 1, 4, 4, 16, 1.0) == INVALID
    for bad in (0, -1):
        assert f(X, X, X, X, X, full, bad, 4, 4, 16, 1.0) == INVALID
        assert f(X, X, X, X, X, full, 1, bad, 4, 16, 1.0) == INVALID
        assert f(X, X, X, X, X, full, 1, 4, 4, 16, 1.0, key_tiles_per_group=bad) == INVALID
    assert f(X, X, X, X, X, full, 1, 4, 4, 16, float("nan")) == INVALID
    # routed (host words given) needs every quantized device buffer
    assert f(X, X, X, X, X, tm.TileMixDeviceBuffers(X, X, X, o=X), 1, 4, 4, 16, 1.0) == INVALID
    assert f(X, X, X, X, X, full, 1, 4, 4, 129, 1.0) == NOT_SUPPORTED


def test_strided_output_validation_without_cuda():
    """tilemix_attention_batched_out rejects bad output layouts before any CUDA call."""
    x = ctypes.create_string_buffer(64)
    X = ctypes.addressof(x)
    f = tm.tilemix_attention_batched_out
    ok = tm.TileMixOutput(X, tm.kTileMixOutF16, 2, 0, 0, 0)
    assert f(X, X, X, None, 2, 4, 4, 16, 1.0) == INVALID
    assert f(X, X, X, tm.TileMixOutput(None, 1, 2), 2, 4, 4, 16, 1.0) == INVALID
    for dtype in (-1, 3):
        assert f(X, X, X, tm.TileMixOutput(X, dtype, 2), 2, 4, 4, 16, 1.0) == INVALID
    assert f(X, X, X, tm.TileMixOutput(X, 1, 0), 2, 4, 4, 16, 1.0) == INVALID
    assert f(X, X, X, tm.TileMixOutput(X, 1, 3), 2, 4, 4, 16, 1.0) == INVALID      # 3 does not divide 2
    for strides in ((-1, 0, 0), (0, -1, 0), (0, 0, -1)):
        assert f(X, X, X, tm.TileMixOutput(X, 1, 2, *strides), 2, 4, 4, 16, 1.0) == INVALID
    assert f(X, X, X, ok, 2, 4, 4, 129, 1.0) == NOT_SUPPORTED
    # trace outputs are not available with a strided output
    quant = tm.TileMixQuantized(X, X, X, X, score_dots=X)
    assert f(X, X, X, ok, 2, 4, 4, 16, 1.0, quantized=quant) == NOT_SUPPORTED
