"""Python host mirror of the TileMix drop-in API over libtilemix_b200.so.

The names, argument meaning and error behaviour follow the reference's C++ API
(``include/attention_fused.h:47-72`` of the reference): functions return the
``cudaError_t`` code as an int (0 = success) instead of raising, exactly like the
C++ entry points, and take device tensors (torch CUDA tensors or raw device
addresses). Everything goes through the extern "C" ABI declared in
``include/tilemix_c_api.h``; there is no CPU fallback: every entry point raises
on a machine without the built library. The library is mapped on the first
call, not at import, so pure-Python helpers such as ``workloads`` load no
native code.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libtilemix_b200.so"

# cudaError_t values used by the contract
cudaSuccess = 0
cudaErrorInvalidValue = 1
cudaErrorInvalidConfiguration = 9
cudaErrorNotSupported = 801

kBlockM, kBlockN, kTileK, kThreads, kWarpSize = 16, 32, 16, 64, 32
kFusedMaxHeadDim = 128
kTileMixQQuantRows = 128
kTileMixKQuantRows = 64

_P = ctypes.c_void_p
_I = ctypes.c_int


class _Routing(ctypes.Structure):
    _fields_ = [("words", _P), ("word_count", ctypes.c_size_t),
                ("key_tiles_per_group", _I), ("decoded_bits", _P)]


class _Quantized(ctypes.Structure):
    _fields_ = [("q", _P), ("k", _P), ("q_scales", _P), ("k_scales", _P), ("score_dots", _P)]


class _Output(ctypes.Structure):
    _fields_ = [("data", _P), ("dtype", _I), ("heads_per_batch", _I), ("stride_batch", ctypes.c_longlong),
                ("stride_head", ctypes.c_longlong), ("stride_row", ctypes.c_longlong)]


class _DeviceBuffers(ctypes.Structure):
    _fields_ = [("q", _P), ("k", _P), ("v", _P), ("q8", _P), ("k8", _P), ("q_scales", _P),
                ("k_scales", _P), ("words", _P), ("o", _P)]


def _load():
    if not LIB_PATH.exists():
        raise RuntimeError(f"{LIB_PATH} is not built; run __graft_entry__.build() "
                           "(there is no CPU fallback for the TileMix kernels)")
    lib = ctypes.CDLL(str(LIB_PATH))
    lib.tilemix_abi_version.restype = _I
    lib.tilemix_quantize_qk.argtypes = [_P, _P, _P, _P, _P, _P, _I, _I, _I, _P]
    lib.tilemix_quantize_qk.restype = _I
    lib.tilemix_fused_attention.argtypes = [_P, _P, _P, _P, _I, _I, _I, ctypes.c_float, _P,
                                            ctypes.POINTER(_Routing), ctypes.POINTER(_Quantized)]
    lib.tilemix_fused_attention.restype = _I
    lib.tilemix_quantize_qk_batched.argtypes = [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _P]
    lib.tilemix_quantize_qk_batched.restype = _I
    lib.tilemix_attention_batched.argtypes = [_P, _P, _P, _P, _I, _I, _I, _I, ctypes.c_float, _I,
                                              _P, ctypes.POINTER(_Routing),
                                              ctypes.POINTER(_Quantized)]
    lib.tilemix_attention_batched.restype = _I
    for name in ("tilemix_routing_word_count_c",):
        getattr(lib, name).argtypes = [_I, _I, _I]
        getattr(lib, name).restype = ctypes.c_size_t
    lib.tilemix_routing_words_per_row_c.argtypes = [_I, _I]
    lib.tilemix_routing_words_per_row_c.restype = ctypes.c_size_t
    lib.tilemix_reference_shared_bytes.argtypes = [_I, _I]
    lib.tilemix_reference_shared_bytes.restype = ctypes.c_size_t
    lib.tilemix_b200_shared_bytes_c.argtypes = [_I, _I]
    lib.tilemix_b200_shared_bytes_c.restype = ctypes.c_size_t
    lib.tilemix_attention_batched_out.argtypes = [_P, _P, _P, ctypes.POINTER(_Output), _I, _I, _I, _I,
                                                  ctypes.c_float, _I, _P, ctypes.POINTER(_Routing),
                                                  ctypes.POINTER(_Quantized)]
    lib.tilemix_attention_batched_out.restype = _I
    lib.tilemix_attention_from_host.argtypes = [_P, _P, _P, _P, _P, ctypes.POINTER(_DeviceBuffers),
                                                _I, _I, _I, _I, ctypes.c_float, _I, _I, _I, _P]
    lib.tilemix_attention_from_host.restype = _I
    lib.tilemix_attention_routed_noalloc.argtypes = [_P, _P, _P, _P, _I, _I, _I, _I, ctypes.c_float, _I,
                                                     ctypes.POINTER(_Routing), _P]
    lib.tilemix_attention_routed_noalloc.restype = _I
    lib.tilemix_quantize_k_batched.argtypes = [_P, _P, _P, _I, _I, _I, _P]
    lib.tilemix_quantize_k_batched.restype = _I
    lib.tilemix_attention_batched_qfused.argtypes = [_P, _P, _P, _P, _I, _I, _I, _I, ctypes.c_float, _I, _P,
                                                     ctypes.POINTER(_Routing), _P, _P, _P, _P]
    lib.tilemix_attention_batched_qfused.restype = _I
    lib.tilemix_quantize_qkv_batched.argtypes = [_P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _P]
    lib.tilemix_quantize_qkv_batched.restype = _I
    lib.tilemix_attention_batched_hinted.argtypes = [_P, _P, _P, _P, _I, _I, _I, _I, ctypes.c_float, _I, _P,
                                                     ctypes.POINTER(_Routing), ctypes.POINTER(_Quantized), _P]
    lib.tilemix_attention_batched_hinted.restype = _I
    lib.tilemix_routing_policy_c.argtypes = [_P, _P, _P, _I, _I, _I, _I, ctypes.c_float, _P]
    lib.tilemix_routing_policy_c.restype = _I
    lib.tilemix_policy_max_scale_product_c.argtypes = [ctypes.c_float, ctypes.c_float, _I]
    lib.tilemix_policy_max_scale_product_c.restype = ctypes.c_float
    lib.tilemix_watchdog_selftest.argtypes = [_P, _P, _P, _P, _I, _I, _I, _I, ctypes.c_float, ctypes.c_uint, _P]
    lib.tilemix_watchdog_selftest.restype = _I
    lib.tilemix_read_and_clear_status.argtypes = [ctypes.POINTER(ctypes.c_uint)]
    lib.tilemix_read_and_clear_status.restype = _I
    lib.tilemix_attention_backward_c.argtypes = [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I,
                                                 ctypes.c_float, _I, _I, _P]
    lib.tilemix_attention_backward_c.restype = _I
    lib.tilemix_attention_batched_lse_c.argtypes = [_P, _P, _P, _P, _P, _I, _I, _I, _I, ctypes.c_float, _I, _P]
    lib.tilemix_attention_batched_lse_c.restype = _I
    lib.tilemix_backward_watchdog_selftest.argtypes = [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I,
                                                       ctypes.c_float, ctypes.c_uint, _P]
    lib.tilemix_backward_watchdog_selftest.restype = _I
    return lib


_lib = None


def _native():
    """The loaded libtilemix_b200.so. Loaded on first use, so that importing the
    package (or its pure-Python helpers such as ``workloads``) maps no native
    code; a call on a machine without the built library raises."""
    global _lib
    if _lib is None:
        _lib = _load()
    return _lib


def __getattr__(name):
    if name == "lib":
        return _native()
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")


# every symbol include/tilemix_c_api.h declares
C_ABI_SYMBOLS = (
    "tilemix_abi_version", "tilemix_quantize_qk", "tilemix_fused_attention",
    "tilemix_quantize_qk_batched", "tilemix_attention_batched", "tilemix_attention_batched_out",
    "tilemix_attention_from_host", "tilemix_attention_routed_noalloc",
    "tilemix_quantize_k_batched", "tilemix_attention_batched_qfused",
    "tilemix_routing_policy_c", "tilemix_policy_max_scale_product_c",
    "tilemix_quantize_qkv_batched", "tilemix_attention_batched_hinted",
    "tilemix_routing_word_count_c", "tilemix_routing_words_per_row_c",
    "tilemix_reference_shared_bytes", "tilemix_b200_shared_bytes_c",
    "tilemix_read_and_clear_status", "tilemix_watchdog_selftest", "tilemix_attention_backward_c",
    "tilemix_attention_batched_lse_c", "tilemix_backward_watchdog_selftest",
)


def _addr(x) -> int | None:
    """Device address of a torch tensor / raw int / None."""
    if x is None:
        return None
    if isinstance(x, int):
        return x or None
    return x.data_ptr() or None


def _stream(stream) -> int | None:
    if stream is None:
        return None
    if isinstance(stream, int):
        return stream or None
    return stream.cuda_stream or None


@dataclass
class TileMixRouting:
    """Routing mask (reference include/attention_fused.h:47-52): one bit per
    (16-row query tile, group of ``key_tiles_per_group`` 32-key tiles); bit 1 = INT8."""
    words: object = None
    word_count: int = 0
    key_tiles_per_group: int = 1
    decoded_bits: object = None

    def _c(self) -> _Routing:
        return _Routing(_addr(self.words), int(self.word_count), int(self.key_tiles_per_group),
                        _addr(self.decoded_bits))


@dataclass
class TileMixQuantized:
    """Quantized operands (reference include/attention_fused.h:54-60)."""
    q: object = None
    k: object = None
    q_scales: object = None
    k_scales: object = None
    score_dots: object = None

    def _c(self) -> _Quantized:
        return _Quantized(_addr(self.q), _addr(self.k), _addr(self.q_scales),
                          _addr(self.k_scales), _addr(self.score_dots))


def tilemix_routing_words_per_row(n: int, key_tiles_per_group: int) -> int:
    return int(_native().tilemix_routing_words_per_row_c(n, key_tiles_per_group))


def tilemix_routing_word_count(m: int, n: int, key_tiles_per_group: int) -> int:
    return int(_native().tilemix_routing_word_count_c(m, n, key_tiles_per_group))


def tilemix_shared_bytes(d: int, quantized: bool) -> int:
    return int(_native().tilemix_reference_shared_bytes(d, int(quantized)))


def tilemix_b200_shared_bytes(d: int, quantized: bool = True) -> int:
    return int(_native().tilemix_b200_shared_bytes_c(d, int(quantized)))


def quantize_tilemix_qk(Q, K, Q8, K8, q_scales, k_scales, M: int, N: int, d: int,
                        stream=None) -> int:
    """Stage 1 (reference src/tilemix.cu:223-236). Returns a cudaError_t code."""
    return _native().tilemix_quantize_qk(_addr(Q), _addr(K), _addr(Q8), _addr(K8), _addr(q_scales),
                                         _addr(k_scales), M, N, d, _stream(stream))


def launch_fused_fp16_attention(Q, K, V, O, M: int, N: int, d: int, score_scale: float,
                                stream=None, routing: TileMixRouting | None = None,
                                quantized: TileMixQuantized | None = None) -> int:
    """Stages 2-5 (reference src/tilemix.cu:238-278). Returns a cudaError_t code."""
    r = (routing or TileMixRouting())._c()
    q = (quantized or TileMixQuantized())._c()
    return _native().tilemix_fused_attention(_addr(Q), _addr(K), _addr(V), _addr(O), M, N, d,
                                             float(score_scale), _stream(stream), ctypes.byref(r),
                                             ctypes.byref(q))


def quantize_tilemix_qk_batched(Q, K, Q8, K8, q_scales, k_scales, heads: int, M: int, N: int,
                                d: int, stream=None) -> int:
    return _native().tilemix_quantize_qk_batched(_addr(Q), _addr(K), _addr(Q8), _addr(K8),
                                                 _addr(q_scales), _addr(k_scales), heads, M, N, d,
                                                 _stream(stream))


def tilemix_attention_batched(Q, K, V, O, heads: int, M: int, N: int, d: int,
                              score_scale: float, causal: bool = False, stream=None,
                              routing: TileMixRouting | None = None,
                              quantized: TileMixQuantized | None = None) -> int:
    r = (routing or TileMixRouting())._c()
    q = (quantized or TileMixQuantized())._c()
    return _native().tilemix_attention_batched(_addr(Q), _addr(K), _addr(V), _addr(O), heads, M, N, d,
                                               float(score_scale), int(bool(causal)), _stream(stream),
                                               ctypes.byref(r), ctypes.byref(q))


def quantize_tilemix_k_batched(K, K8, k_scales, heads: int, N: int, d: int, stream=None) -> int:
    """K alone in 64-row blocks (the K half of quantize_tilemix_qk_batched)."""
    return _native().tilemix_quantize_k_batched(_addr(K), _addr(K8), _addr(k_scales), heads, N, d, _stream(stream))


def tilemix_attention_batched_qfused(Q, K, V, O, heads: int, M: int, N: int, d: int, score_scale: float,
                                     causal: bool = False, stream=None, routing: TileMixRouting | None = None,
                                     K8=None, k_scales=None, Q8_out=None, q_scales_out=None) -> int:
    """Routed attention with Q quantized inside the attention kernel (one HBM
    pass over Q fewer). Routing words, K8 and k_scales are required; Q8_out /
    q_scales_out optionally receive the bytes the standalone quantizer makes."""
    r = (routing or TileMixRouting())._c()
    return _native().tilemix_attention_batched_qfused(_addr(Q), _addr(K), _addr(V), _addr(O), heads, M, N, d,
                                                      float(score_scale), int(bool(causal)), _stream(stream),
                                                      ctypes.byref(r), _addr(K8), _addr(k_scales), _addr(Q8_out),
                                                      _addr(q_scales_out))


def quantize_tilemix_qkv_batched(Q, K, V, Q8, K8, q_scales, k_scales, v_absmax, heads: int, M: int, N: int,
                                 d: int, stream=None) -> int:
    """quantize_tilemix_qk_batched plus max |v| per 64-row V block (fp16
    [heads, ceil(N/64)]) in the same launch."""
    return _native().tilemix_quantize_qkv_batched(_addr(Q), _addr(K), _addr(V), _addr(Q8), _addr(K8),
                                                  _addr(q_scales), _addr(k_scales), _addr(v_absmax), heads, M, N,
                                                  d, _stream(stream))


def tilemix_attention_batched_hinted(Q, K, V, O, heads: int, M: int, N: int, d: int, score_scale: float,
                                     causal: bool = False, stream=None, routing: TileMixRouting | None = None,
                                     quantized: TileMixQuantized | None = None, v_absmax=None) -> int:
    """tilemix_attention_batched with single-term fp16 P for the 64-key halves
    whose max |v| (v_absmax) is <= 3.5 (at most 1.7e-3 added to any output)."""
    r = (routing or TileMixRouting())._c()
    q = (quantized or TileMixQuantized())._c()
    return _native().tilemix_attention_batched_hinted(_addr(Q), _addr(K), _addr(V), _addr(O), heads, M, N, d,
                                                      float(score_scale), int(bool(causal)), _stream(stream),
                                                      ctypes.byref(r), ctypes.byref(q), _addr(v_absmax))


def tilemix_routing_policy(q_scales, k_scales, words, heads: int, M: int, N: int, key_tiles_per_group: int,
                           max_scale_product: float, stream=None) -> int:
    """Routing words from the quantizer's block scales: INT8 iff q_scale *
    max k_scale of the key group <= max_scale_product (fp32), else FP16."""
    return _native().tilemix_routing_policy_c(_addr(q_scales), _addr(k_scales), _addr(words), heads, M, N,
                                              key_tiles_per_group, float(max_scale_product), _stream(stream))


def tilemix_policy_max_scale_product(tolerance: float, score_scale: float, d: int) -> float:
    """The product threshold that bounds the INT8 score error by `tolerance`:
    tolerance / (|score_scale| * d * 127.25)."""
    return float(_native().tilemix_policy_max_scale_product_c(float(tolerance), float(score_scale), int(d)))


kTileMixOutF32, kTileMixOutF16, kTileMixOutBF16 = 0, 1, 2


@dataclass
class TileMixOutput:
    """Strided output (include/attention_fused.h TileMixOutput): head
    h = b * heads_per_batch + hh, row m, column c at data + b * stride_batch +
    hh * stride_head + m * stride_row + c, in elements of `dtype`."""
    data: object = None
    dtype: int = kTileMixOutF32
    heads_per_batch: int = 1
    stride_batch: int = 0
    stride_head: int = 0
    stride_row: int = 0

    def _c(self) -> _Output:
        return _Output(_addr(self.data), int(self.dtype), int(self.heads_per_batch), int(self.stride_batch),
                       int(self.stride_head), int(self.stride_row))

    @classmethod
    def bshd(cls, tensor, heads_per_batch: int):
        """A [B, S, H, D] torch tensor (fp32 / fp16 / bf16, contiguous or strided)."""
        import torch
        dt = {torch.float32: kTileMixOutF32, torch.float16: kTileMixOutF16,
              torch.bfloat16: kTileMixOutBF16}[tensor.dtype]
        sb, ss, sh, sd = tensor.stride()
        if sd != 1:
            raise ValueError("the head dimension must be contiguous")
        return cls(tensor, dt, heads_per_batch, sb, sh, ss)


def tilemix_attention_batched_out(Q, K, V, out: TileMixOutput | None, heads: int, M: int, N: int, d: int,
                                  score_scale: float, causal: bool = False, stream=None,
                                  routing: TileMixRouting | None = None,
                                  quantized: TileMixQuantized | None = None) -> int:
    """tilemix_attention_batched writing O through a strided fp32/fp16/bf16 output."""
    r = (routing or TileMixRouting())._c()
    q = (quantized or TileMixQuantized())._c()
    o = out._c() if out is not None else None
    return _native().tilemix_attention_batched_out(_addr(Q), _addr(K), _addr(V),
                                                   ctypes.byref(o) if o is not None else None, heads, M, N, d,
                                                   float(score_scale), int(bool(causal)), _stream(stream),
                                                   ctypes.byref(r), ctypes.byref(q))


def _host_addr(x) -> int | None:
    """Host address of a CPU torch tensor / numpy array / raw int / None."""
    if x is None:
        return None
    if isinstance(x, int):
        return x or None
    if hasattr(x, "data_ptr"):
        return x.data_ptr() or None
    return x.ctypes.data or None


@dataclass
class TileMixDeviceBuffers:
    """Device buffers of tilemix_attention_from_host, sized for all heads."""
    q: object = None
    k: object = None
    v: object = None
    q8: object = None
    k8: object = None
    q_scales: object = None
    k_scales: object = None
    words: object = None
    o: object = None

    def _c(self) -> _DeviceBuffers:
        return _DeviceBuffers(*(_addr(getattr(self, f)) for f, _ in _DeviceBuffers._fields_))


def tilemix_attention_from_host(hQ, hK, hV, h_words, hO, dev: TileMixDeviceBuffers, heads: int,
                                M: int, N: int, d: int, score_scale: float, causal: bool = False,
                                key_tiles_per_group: int = 2, chunk_heads: int = 0,
                                stream=None) -> int:
    """H2D copies, quantization, routed attention and the D2H copy of O for
    host (pinned) buffers, pipelined over chunks of heads. Returns a cudaError_t code."""
    b = dev._c() if dev is not None else None
    return _native().tilemix_attention_from_host(_host_addr(hQ), _host_addr(hK), _host_addr(hV),
                                                 _host_addr(h_words), _host_addr(hO),
                                                 ctypes.byref(b) if b is not None else None,
                                                 heads, M, N, d, float(score_scale), int(bool(causal)),
                                                 key_tiles_per_group, chunk_heads, _stream(stream))


# Size of the library's fixed device scratch used by
# tilemix_attention_routed_noalloc (TILEMIX_NOALLOC_SCRATCH_BYTES).
NOALLOC_SCRATCH_BYTES = 64 << 20
cudaErrorMemoryAllocation = 2


def tilemix_attention_routed_noalloc(Q, K, V, O, heads: int, M: int, N: int, d: int, score_scale: float,
                                     causal: bool = False, routing: TileMixRouting | None = None,
                                     stream=None) -> int:
    """Quantization and routed attention with the INT8 Q/K copies and their
    scales in the library's fixed device scratch, for callers that cannot
    allocate device memory (they pass only Q, K, V, the routing words and O).
    Problems whose INT8 copies exceed NOALLOC_SCRATCH_BYTES return
    cudaErrorMemoryAllocation; calls that overlap on the GPU share the scratch
    and race. Returns a cudaError_t code."""
    r = (routing or TileMixRouting())._c()
    return _native().tilemix_attention_routed_noalloc(_addr(Q), _addr(K), _addr(V), _addr(O), heads, M, N, d,
                                                      float(score_scale), int(bool(causal)), ctypes.byref(r),
                                                      _stream(stream))


# watchdog status bits (which kind of wait gave up): forward kernel roles,
# then the backward kernels' pipeline waits and drains
STATUS_PRODUCER, STATUS_MMA, STATUS_SOFTMAX, STATUS_DRAIN = 1, 2, 4, 8
STATUS_BACKWARD_WAIT, STATUS_BACKWARD_DRAIN = 16, 32


def watchdog_selftest(Q, K, V, O, heads: int, M: int, N: int, d: int, score_scale: float,
                      wait_limit_us: int, stream=None) -> int:
    """Run the kernel build that withholds one P-ready arrival per CTA, with
    waits limited to wait_limit_us; the watchdog must record STATUS_MMA and
    the kernel return. O is not valid afterwards. Returns a cudaError_t code."""
    return _native().tilemix_watchdog_selftest(_addr(Q), _addr(K), _addr(V), _addr(O), heads, M, N, d,
                                               float(score_scale), int(wait_limit_us), _stream(stream))


def tilemix_attention_batched_lse(Q, K, V, O, lse, heads: int, M: int, N: int, d: int, score_scale: float,
                                  causal: bool = False, stream=None) -> int:
    """Unrouted attention that also writes each row's base-2 log-sum-exp
    (fp32 [heads, M]) for the backward pass. Returns a cudaError_t code."""
    return _native().tilemix_attention_batched_lse_c(_addr(Q), _addr(K), _addr(V), _addr(O), _addr(lse), heads, M,
                                                     N, d, float(score_scale), int(bool(causal)), _stream(stream))


def tilemix_attention_backward(Q, K, V, O, dO, dQ, dK, dV, lse, dsum, heads: int, M: int, N: int, d: int,
                               score_scale: float, causal: bool = False, stream=None,
                               lse_from_forward: bool = False) -> int:
    """Backward of the unrouted attention through the C-ABI: fp16 Q, K, V, dO,
    fp32 O (the forward's output), fp32 dQ, dK, dV outputs, fp32 [heads, M]
    lse / dsum (lse read when lse_from_forward, else written). Returns a
    cudaError_t code."""
    return _native().tilemix_attention_backward_c(_addr(Q), _addr(K), _addr(V), _addr(O), _addr(dO), _addr(dQ),
                                                  _addr(dK), _addr(dV), _addr(lse), _addr(dsum), heads, M, N, d,
                                                  float(score_scale), int(bool(causal)), int(bool(lse_from_forward)),
                                                  _stream(stream))


def backward_watchdog_selftest(Q, K, V, O, dO, dQ, dK, dV, lse, dsum, heads: int, M: int, N: int, d: int,
                               score_scale: float, wait_limit_us: int, stream=None) -> int:
    """The backward with its column kernel built to withhold one P-ready
    arrival per CTA, waits limited to wait_limit_us: the watchdog must record
    STATUS_BACKWARD_WAIT and the kernels return. The gradients are not valid
    afterwards. Returns a cudaError_t code."""
    return _native().tilemix_backward_watchdog_selftest(_addr(Q), _addr(K), _addr(V), _addr(O), _addr(dO),
                                                        _addr(dQ), _addr(dK), _addr(dV), _addr(lse), _addr(dsum),
                                                        heads, M, N, d, float(score_scale), int(wait_limit_us),
                                                        _stream(stream))


def read_and_clear_status() -> tuple[int, int]:
    """(cudaError_t, watchdog word) of the current device; synchronises."""
    s = ctypes.c_uint(0)
    err = _native().tilemix_read_and_clear_status(ctypes.byref(s))
    return err, int(s.value)


class TileMixError(RuntimeError):
    pass


def check(err: int, what: str = "tilemix call") -> None:
    if err != cudaSuccess:
        raise TileMixError(f"{what} failed with cudaError_t {err}")


# ------------------------------------------------- torch convenience wrappers
def _current_stream(t):
    """torch's current stream on t's device (the kernels are ordered with the
    producers and consumers of t), as a raw cudaStream_t."""
    import torch
    return torch.cuda.current_stream(t.device).cuda_stream


def _require(cond: bool, msg: str) -> None:
    if not cond:
        raise ValueError(msg)


def _heads3_shape(t, name: str):
    _require(t.dim() in (2, 3), f"{name} must be [S, d] or [heads, S, d], got shape {tuple(t.shape)}")
    return tuple(t.shape) if t.dim() == 3 else (1, *t.shape)


def _on_device(t, like, device_check: bool) -> bool:
    return not device_check or (t.is_cuda and t.device == like.device)


def validate_quantize_args(q, k, device_check: bool = True) -> tuple[int, int, int, int]:
    """Checks the tensors of a quantization call before any device pointer is
    taken: fp16 CUDA tensors on one device, q [heads, M, d] and k [heads, N, d]
    with equal heads and d (the kernel takes heads and d from q, so a smaller k
    would be read past its end). Raises ValueError; returns (heads, M, N, d).
    device_check=False skips the CUDA-device checks (shape checks on meta
    tensors)."""
    import torch
    for t, name in ((q, "q"), (k, "k")):
        _require(isinstance(t, torch.Tensor) and _on_device(t, q, device_check), f"{name} must be a CUDA tensor")
        _require(t.dtype == torch.float16, f"{name} must be float16, got {t.dtype}")
    _require(q.dim() == k.dim(), "q and k must have the same number of dimensions")
    heads, m, d = _heads3_shape(q, "q")
    kh, n, kd = _heads3_shape(k, "k")
    _require(kh == heads and kd == d, f"k {tuple(k.shape)} does not match q {tuple(q.shape)} in heads and d")
    return heads, m, n, d


def validate_attention_args(q, k, v, q8=None, k8=None, q_scales=None, k_scales=None, words=None,
                            key_tiles_per_group: int = 2, device_check: bool = True) -> tuple[int, int, int, int]:
    """Checks dtypes, devices and cross-tensor shapes of an attention call:
    q [heads, M, d], k and v [heads, N, d] fp16; q8/k8 int8 of q's/k's shape;
    scales fp16 with heads * ceil(M/128) and heads * ceil(N/64) elements; the
    routing words 64-bit with at least heads * tilemix_routing_word_count
    elements. The C-ABI checks the scalar arguments; these checks keep it from
    reading past the end of a tensor whose shape disagrees with q's.
    Returns (heads, M, N, d)."""
    import torch
    heads, m, n, d = validate_quantize_args(q, k, device_check)
    _require(isinstance(v, torch.Tensor) and _on_device(v, q, device_check), "v must be a CUDA tensor on q's device")
    _require(v.dtype == torch.float16, f"v must be float16, got {v.dtype}")
    _require(tuple(v.shape) == tuple(k.shape), f"v {tuple(v.shape)} must have k's shape {tuple(k.shape)}")
    quant = (q8, k8, q_scales, k_scales)
    if any(t is not None for t in quant):
        _require(all(t is not None for t in quant), "q8, k8, q_scales and k_scales go together")
        for t, name, dt, shape in ((q8, "q8", torch.int8, None), (k8, "k8", torch.int8, None),
                                   (q_scales, "q_scales", torch.float16, heads * ((m - 1) // 128 + 1)),
                                   (k_scales, "k_scales", torch.float16, heads * ((n - 1) // 64 + 1))):
            _require(_on_device(t, q, device_check), f"{name} must be a CUDA tensor on q's device")
            _require(t.dtype == dt, f"{name} must be {dt}, got {t.dtype}")
            if shape is not None:
                _require(t.numel() == shape, f"{name} must hold {shape} elements, got {t.numel()}")
        _require(tuple(q8.shape) == tuple(q.shape), f"q8 {tuple(q8.shape)} must have q's shape")
        _require(tuple(k8.shape) == tuple(k.shape), f"k8 {tuple(k8.shape)} must have k's shape")
    if words is not None:
        _require(_on_device(words, q, device_check), "words must be a CUDA tensor on q's device")
        _require(words.dtype in (torch.int64, torch.uint64), f"words must be 64-bit, got {words.dtype}")
        _require(q8 is not None, "routing words need the quantized operands (q8, k8, q_scales, k_scales)")
        need = heads * tilemix_routing_word_count(m, n, key_tiles_per_group)
        _require(words.numel() >= need, f"words must hold at least {need} elements, got {words.numel()}")
    return heads, m, n, d


def quantize(q, k, stream=None):
    """Allocate outputs and quantize [heads,M,d] / [heads,N,d] (or 2-D) fp16
    CUDA tensors. Returns (q8, k8, q_scales, k_scales). Runs on torch's current
    stream of q's device unless `stream` is given."""
    import torch
    heads, m, n, d = validate_quantize_args(q, k)
    q, k = q.contiguous(), k.contiguous()
    q8 = torch.empty_like(q, dtype=torch.int8)
    k8 = torch.empty_like(k, dtype=torch.int8)
    qs = torch.empty((heads, (m - 1) // 128 + 1), dtype=torch.float16, device=q.device)
    ks = torch.empty((heads, (n - 1) // 64 + 1), dtype=torch.float16, device=q.device)
    check(quantize_tilemix_qk_batched(q, k, q8, k8, qs, ks, heads, m, n, d,
                                      _current_stream(q) if stream is None else stream), "quantize")
    if q.dim() == 2:
        qs, ks = qs[0], ks[0]
    return q8, k8, qs, ks


def attention(q, k, v, *, q8=None, k8=None, q_scales=None, k_scales=None, words=None,
              key_tiles_per_group: int = 2, score_scale: float | None = None,
              causal: bool = False, out=None, stream=None):
    """[heads,M,d] (or 2-D) fp16 CUDA tensors -> fp32 output through the C-ABI.
    Runs on torch's current stream of q's device unless `stream` is given."""
    import torch
    heads, m, n, d = validate_attention_args(q, k, v, q8, k8, q_scales, k_scales, words, key_tiles_per_group)
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    if q8 is not None:
        q8, k8, q_scales, k_scales = (t.contiguous() for t in (q8, k8, q_scales, k_scales))
    if words is not None:
        words = words.contiguous()
    if score_scale is None:
        score_scale = 1.0 / math.sqrt(d)
    if out is None:
        out = torch.empty(q.shape, dtype=torch.float32, device=q.device)
    else:
        _require(out.is_cuda and out.device == q.device and out.dtype == torch.float32 and
                 tuple(out.shape) == tuple(q.shape) and out.is_contiguous(),
                 "out must be a contiguous float32 CUDA tensor of q's shape on q's device")
    routing = TileMixRouting(words, 0 if words is None else words.numel(), key_tiles_per_group)
    quantized = TileMixQuantized(q8, k8, q_scales, k_scales) if q8 is not None else None
    check(tilemix_attention_batched(q, k, v, out, heads, m, n, d, score_scale, causal,
                                    _current_stream(q) if stream is None else stream, routing, quantized),
          "attention")
    return out
