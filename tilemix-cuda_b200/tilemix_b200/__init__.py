"""Python host mirror of the TileMix drop-in API over libtilemix_b200.so.

The names, argument meaning and error behaviour follow the reference's C++ API
(``include/attention_fused.h:47-72`` of the reference): functions return the
``cudaError_t`` code as an int (0 = success) instead of raising, exactly like the
C++ entry points, and take device tensors (torch CUDA tensors or raw device
addresses). Everything goes through the extern "C" ABI declared in
``include/tilemix_c_api.h``; there is no CPU fallback: importing this module on a
machine without the built library raises.
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
    lib.tilemix_read_and_clear_status.argtypes = [ctypes.POINTER(ctypes.c_uint)]
    lib.tilemix_read_and_clear_status.restype = _I
    return lib


lib = _load()

# every symbol include/tilemix_c_api.h declares
C_ABI_SYMBOLS = (
    "tilemix_abi_version", "tilemix_quantize_qk", "tilemix_fused_attention",
    "tilemix_quantize_qk_batched", "tilemix_attention_batched", "tilemix_attention_batched_out",
    "tilemix_attention_from_host",
    "tilemix_routing_word_count_c", "tilemix_routing_words_per_row_c",
    "tilemix_reference_shared_bytes", "tilemix_b200_shared_bytes_c",
    "tilemix_read_and_clear_status",
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
    return int(lib.tilemix_routing_words_per_row_c(n, key_tiles_per_group))


def tilemix_routing_word_count(m: int, n: int, key_tiles_per_group: int) -> int:
    return int(lib.tilemix_routing_word_count_c(m, n, key_tiles_per_group))


def tilemix_shared_bytes(d: int, quantized: bool) -> int:
    return int(lib.tilemix_reference_shared_bytes(d, int(quantized)))


def tilemix_b200_shared_bytes(d: int, quantized: bool = True) -> int:
    return int(lib.tilemix_b200_shared_bytes_c(d, int(quantized)))


def quantize_tilemix_qk(Q, K, Q8, K8, q_scales, k_scales, M: int, N: int, d: int,
                        stream=None) -> int:
    """Stage 1 (reference src/tilemix.cu:223-236). Returns a cudaError_t code."""
    return lib.tilemix_quantize_qk(_addr(Q), _addr(K), _addr(Q8), _addr(K8), _addr(q_scales),
                                   _addr(k_scales), M, N, d, _stream(stream))


def launch_fused_fp16_attention(Q, K, V, O, M: int, N: int, d: int, score_scale: float,
                                stream=None, routing: TileMixRouting | None = None,
                                quantized: TileMixQuantized | None = None) -> int:
    """Stages 2-5 (reference src/tilemix.cu:238-278). Returns a cudaError_t code."""
    r = (routing or TileMixRouting())._c()
    q = (quantized or TileMixQuantized())._c()
    return lib.tilemix_fused_attention(_addr(Q), _addr(K), _addr(V), _addr(O), M, N, d,
                                       float(score_scale), _stream(stream), ctypes.byref(r),
                                       ctypes.byref(q))


def quantize_tilemix_qk_batched(Q, K, Q8, K8, q_scales, k_scales, heads: int, M: int, N: int,
                                d: int, stream=None) -> int:
    return lib.tilemix_quantize_qk_batched(_addr(Q), _addr(K), _addr(Q8), _addr(K8),
                                           _addr(q_scales), _addr(k_scales), heads, M, N, d,
                                           _stream(stream))


def tilemix_attention_batched(Q, K, V, O, heads: int, M: int, N: int, d: int,
                              score_scale: float, causal: bool = False, stream=None,
                              routing: TileMixRouting | None = None,
                              quantized: TileMixQuantized | None = None) -> int:
    r = (routing or TileMixRouting())._c()
    q = (quantized or TileMixQuantized())._c()
    return lib.tilemix_attention_batched(_addr(Q), _addr(K), _addr(V), _addr(O), heads, M, N, d,
                                         float(score_scale), int(bool(causal)), _stream(stream),
                                         ctypes.byref(r), ctypes.byref(q))


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
    return lib.tilemix_attention_batched_out(_addr(Q), _addr(K), _addr(V),
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
    return lib.tilemix_attention_from_host(_host_addr(hQ), _host_addr(hK), _host_addr(hV),
                                           _host_addr(h_words), _host_addr(hO),
                                           ctypes.byref(b) if b is not None else None,
                                           heads, M, N, d, float(score_scale), int(bool(causal)),
                                           key_tiles_per_group, chunk_heads, _stream(stream))


def read_and_clear_status() -> tuple[int, int]:
    """(cudaError_t, watchdog word) of the current device; synchronises."""
    s = ctypes.c_uint(0)
    err = lib.tilemix_read_and_clear_status(ctypes.byref(s))
    return err, int(s.value)


class TileMixError(RuntimeError):
    pass


def check(err: int, what: str = "tilemix call") -> None:
    if err != cudaSuccess:
        raise TileMixError(f"{what} failed with cudaError_t {err}")


# ------------------------------------------------- torch convenience wrappers
def quantize(q, k, stream=None):
    """Allocate outputs and quantize [heads,M,d] / [heads,N,d] (or 2-D) fp16
    CUDA tensors. Returns (q8, k8, q_scales, k_scales)."""
    import torch
    q3 = q if q.dim() == 3 else q.unsqueeze(0)
    k3 = k if k.dim() == 3 else k.unsqueeze(0)
    heads, m, d = q3.shape
    n = k3.shape[1]
    q8 = torch.empty_like(q, dtype=torch.int8)
    k8 = torch.empty_like(k, dtype=torch.int8)
    qs = torch.empty((heads, (m - 1) // 128 + 1), dtype=torch.float16, device=q.device)
    ks = torch.empty((heads, (n - 1) // 64 + 1), dtype=torch.float16, device=q.device)
    check(quantize_tilemix_qk_batched(q, k, q8, k8, qs, ks, heads, m, n, d, stream), "quantize")
    if q.dim() == 2:
        qs, ks = qs[0], ks[0]
    return q8, k8, qs, ks


def attention(q, k, v, *, q8=None, k8=None, q_scales=None, k_scales=None, words=None,
              key_tiles_per_group: int = 2, score_scale: float | None = None,
              causal: bool = False, out=None, stream=None):
    """[heads,M,d] (or 2-D) fp16 CUDA tensors -> fp32 output through the C-ABI."""
    import torch
    q3 = q if q.dim() == 3 else q.unsqueeze(0)
    heads, m, d = q3.shape
    n = (k if k.dim() == 3 else k.unsqueeze(0)).shape[1]
    if score_scale is None:
        score_scale = 1.0 / math.sqrt(d)
    if out is None:
        out = torch.empty(q.shape, dtype=torch.float32, device=q.device)
    routing = TileMixRouting(words, 0 if words is None else words.numel(), key_tiles_per_group)
    quantized = TileMixQuantized(q8, k8, q_scales, k_scales) if q8 is not None else None
    check(tilemix_attention_batched(q, k, v, out, heads, m, n, d, score_scale, causal, stream,
                                    routing, quantized), "attention")
    return out
