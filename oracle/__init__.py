"""TileMix CPU oracle -- TEST INFRASTRUCTURE ONLY.

Python (ctypes + numpy) access to two CPU checkers:

* ``libtilemix_oracle.so`` -- the plain-C restatement in ``tilemix_oracle.c``
  of the reference's CPU semantics (reference files
  ``src/tests/reference_tilemix.h:16-89``, ``src/tests/reference_attention.h:12-52``,
  ``src/tilemix.cu:16-49,99-103``), extended with batching and a causal mask;
* ``oracle/_ref/libtilemix_ref.so`` -- the reference's OWN CPU oracle headers
  compiled in place by ``oracle/build_ref.sh`` (absent on machines without the
  reference tree; the committed golden vectors under ``tests/golden/`` carry its
  outputs there).

It also loads ``oracle/_ref/libtilemix_ref_gpu.so``, the reference's own GPU
kernels (``src/tilemix.cu``) compiled in place for sm_100a, which only
``bench.py --impl reference`` times (its "reference GPU" column).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
and reference arm may use this package, and only as the checker / the timed
reference. The product library never imports it.
"""
from __future__ import annotations

import ctypes
import json
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "_build" / "libtilemix_oracle.so"
REF_SO = HERE / "_ref" / "libtilemix_ref.so"
REF_GPU_SO = HERE / "_ref" / "libtilemix_ref_gpu.so"

_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float

_lib = None
_ref = None
_ref_gpu = None


def _reference_root() -> Path | None:
    """Where the reference checkout lives, when it is present (build hosts
    only; the prebuilt oracle/_ref libraries travel without it): the
    TILEMIX_REFERENCE_ROOT environment variable, else the `reference_path`
    field of the repository's BASELINE.json. None when neither names one."""
    env = os.environ.get("TILEMIX_REFERENCE_ROOT")
    if env:
        return Path(env)
    baseline = HERE.parent / "BASELINE.json"
    try:
        path = json.loads(baseline.read_text()).get("reference_path")
    except (OSError, ValueError):
        path = None
    return Path(path) if path else None


REFERENCE_ROOT = _reference_root()


def reference_tree_present() -> bool:
    return REFERENCE_ROOT is not None and (REFERENCE_ROOT / "src" / "tests" / "reference_tilemix.h").is_file()


def build(reference_root: str | None = None) -> None:
    """Compile the C oracle (and the reference shim when the tree exists)."""
    root = reference_root or (str(REFERENCE_ROOT) if REFERENCE_ROOT is not None else "")
    cmd = ["bash", str(HERE / "build_ref.sh"), root]
    subprocess.run(cmd, check=True, stdout=subprocess.DEVNULL)


def lib():
    """The C restatement, built on first use if missing."""
    global _lib
    if _lib is None:
        if not ORACLE_SO.exists():
            build()
        _lib = ctypes.CDLL(str(ORACLE_SO))
        _lib.orc_float_to_half.restype = ctypes.c_uint16
        _lib.orc_float_to_half.argtypes = [_F]
        _lib.orc_half_to_float.restype = _F
        _lib.orc_half_to_float.argtypes = [ctypes.c_uint16]
        _lib.orc_int8_dot.restype = ctypes.c_int32
        _lib.orc_int8_dot.argtypes = [_P, _P, _I, _I, _I]
        _lib.orc_decode_routing.restype = _I
        _lib.orc_decode_routing.argtypes = [_P, _I, _I, _I, _P]
        _lib.orc_pack_block_mask64.argtypes = [_P, _I, _I, _P]
        _lib.orc_quantize_rows.argtypes = [_P, _I, _I, _I, _P, _P]
        _lib.orc_quantize_batched.argtypes = [_P, _I, _I, _I, _I, _P, _P]
        _lib.orc_routing_policy.argtypes = [_P, _P, _I, _I, _I, _I, _F, _P]
        _lib.orc_tilemix_batched.argtypes = [_P, _P, _P, _P, _P, _P, _P, _P,
                                             _I, _I, _I, _I, _F, _I, _P]
        _lib.orc_tilemix_sampled.argtypes = [_P, _P, _P, _P, _P, _P, _P, _P,
                                             _I, _I, _I, _F, _I, _P, _I, _P, _I, _P]
        _lib.orc_dense_attention.argtypes = [_P, _P, _P, _I, _I, _I, _P]
        _lib.orc_reference_inputs.argtypes = [_I, _I, _I, _P, _P, _P]
        _lib.orc_max_threads.restype = _I
        _lib.orc_set_threads.argtypes = [_I]
    return _lib


def ref_available() -> bool:
    return REF_SO.exists()


def ref_lib():
    """The reference's own CPU oracle (compiled in place), or None."""
    global _ref
    if _ref is None and REF_SO.exists():
        _ref = ctypes.CDLL(str(REF_SO))
        _ref.ref_quantize.argtypes = [_P, _I, _I, _I, _P, _P]
        _ref.ref_int8_dot.restype = ctypes.c_int32
        _ref.ref_int8_dot.argtypes = [_P, _P, _I, _I, _I, _I, _I]
        _ref.ref_tilemix.argtypes = [_P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _F, _P]
        _ref.ref_attention.argtypes = [_P, _P, _P, _I, _I, _I, _P]
        _ref.ref_tilemix_sampled.argtypes = [_P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _F,
                                             _I, _P, _I, _P, _I, _P]
        _ref.ref_max_threads.restype = _I
        _ref.ref_set_threads.argtypes = [_I]
    return _ref


def ref_gpu_lib():
    """The reference's own GPU kernels (compiled in place for sm_100a), or None."""
    global _ref_gpu
    if _ref_gpu is None and REF_GPU_SO.exists():
        _ref_gpu = ctypes.CDLL(str(REF_GPU_SO))
        _ref_gpu.ref_gpu_tilemix_heads.restype = _I
        _ref_gpu.ref_gpu_tilemix_heads.argtypes = [_P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _F,
                                                   _P, ctypes.c_size_t, _I, _P]
    return _ref_gpu


def _ptr(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(ctypes.c_void_p)


def _u16(a: np.ndarray) -> np.ndarray:
    """fp16 array -> contiguous uint16 bit view."""
    a = np.ascontiguousarray(a)
    if a.dtype == np.float16:
        return a.view(np.uint16)
    assert a.dtype == np.uint16, a.dtype
    return a


# ----------------------------------------------------------------- primitives
def float_to_half_bits(x: np.ndarray) -> np.ndarray:
    f = lib().orc_float_to_half
    flat = np.ascontiguousarray(x, dtype=np.float32).ravel()
    return np.fromiter((f(float(v)) for v in flat), dtype=np.uint16, count=flat.size)


def reference_inputs(m: int, n: int, d: int):
    """The reference test's deterministic inputs (tilemix_test.cu:43-54)."""
    q = np.empty((m, d), np.uint16)
    k = np.empty((n, d), np.uint16)
    v = np.empty((n, d), np.uint16)
    lib().orc_reference_inputs(m, n, d, _ptr(q), _ptr(k), _ptr(v))
    return q.view(np.float16), k.view(np.float16), v.view(np.float16)


def quantize(x: np.ndarray, block_rows: int):
    """Per-block INT8 quantizer. x: [rows, d] or [heads, rows, d] fp16.
    Returns (int8 values shaped like x, fp16 scales [..., ceil(rows/block_rows)])."""
    xb = _u16(x)
    if xb.ndim == 2:
        rows, d = xb.shape
        heads = 1
    else:
        heads, rows, d = xb.shape
    blocks = (rows - 1) // block_rows + 1
    values = np.empty(xb.shape, np.int8)
    scales = np.empty((heads, blocks), np.uint16)
    lib().orc_quantize_batched(_ptr(xb), heads, rows, d, block_rows, _ptr(values), _ptr(scales))
    if xb.ndim == 2:
        scales = scales[0]
    return values, scales.view(np.float16)


def int8_dot(q8: np.ndarray, k8: np.ndarray, query: int, key: int) -> int:
    d = q8.shape[-1]
    return int(lib().orc_int8_dot(_ptr(np.ascontiguousarray(q8)), _ptr(np.ascontiguousarray(k8)),
                                  query, key, d))


def int8_dots(q8: np.ndarray, k8: np.ndarray) -> np.ndarray:
    """All exact INT32 dots [M, N] (vectorised form of int8_dot)."""
    return q8.astype(np.int32) @ k8.astype(np.int32).T


def routing_words_per_row(n: int, g: int) -> int:
    if n <= 0 or g <= 0:
        return 0
    key_tiles = (n - 1) // 32 + 1
    groups = (key_tiles - 1) // g + 1
    return (groups - 1) // 64 + 1


def routing_word_count(m: int, n: int, g: int) -> int:
    if m <= 0:
        return 0
    return ((m - 1) // 16 + 1) * routing_words_per_row(n, g)


def decode_routing(words: np.ndarray | None, m: int, n: int, g: int) -> np.ndarray:
    """Routing words -> uint8 bits [ceil(m/16), ceil(n/32)] (tilemix.cu:99-103)."""
    bits = np.zeros(((m + 15) // 16, (n + 31) // 32), np.uint8)
    w = None if words is None else np.ascontiguousarray(words, dtype=np.uint64)
    rc = lib().orc_decode_routing(_ptr(w), m, n, g, _ptr(bits))
    assert rc == 0
    return bits


def pack_block_mask64(block_mask: np.ndarray, m: int, n: int) -> np.ndarray:
    """[ceil(m/64), ceil(n/64)] 0/1 mask -> reference words with g=2."""
    bm = np.ascontiguousarray(block_mask, dtype=np.uint8)
    words = np.zeros(routing_word_count(m, n, 2), np.uint64)
    lib().orc_pack_block_mask64(_ptr(bm), m, n, _ptr(words))
    return words


# ------------------------------------------------------------------ attention
def _batched(a):
    return a if a.ndim == 3 else a[None]


def tilemix_attention(q, k, v, q8=None, k8=None, q_scales=None, k_scales=None, routes=None,
                      score_scale: float | None = None, causal: bool = False) -> np.ndarray:
    """Mixed INT8/FP16 attention in fp64 (reference_tilemix.h:53-89).
    Inputs [M,d] or [heads,M,d]; routes [.., ceil(M/16), ceil(N/32)] uint8 or None."""
    squeeze = q.ndim == 2
    q, k, v = (_u16(_batched(t)) for t in (q, k, v))
    heads, m, d = q.shape
    n = k.shape[1]
    if score_scale is None:
        score_scale = 1.0 / np.sqrt(np.float32(d))
    args = []
    for t in (q8, k8):
        args.append(None if t is None else np.ascontiguousarray(_batched(t), dtype=np.int8))
    for t in (q_scales, k_scales):
        args.append(None if t is None else _u16(np.asarray(t).reshape(heads, -1)))
    r = None if routes is None else np.ascontiguousarray(routes, dtype=np.uint8).reshape(heads, -1)
    out = np.empty((heads, m, d), np.float64)
    lib().orc_tilemix_batched(_ptr(q), _ptr(k), _ptr(v), _ptr(args[0]), _ptr(args[1]),
                              _ptr(args[2]), _ptr(args[3]), _ptr(r), heads, m, n, d,
                              float(score_scale), int(causal), _ptr(out))
    return out[0] if squeeze else out


def tilemix_sampled(q, k, v, q8, k8, q_scales, k_scales, routes, head_ids, row_ids,
                    score_scale: float, causal: bool, use_reference: bool = False) -> np.ndarray:
    """Selected rows of selected heads; returns [len(head_ids), len(row_ids), d] fp64.
    use_reference=True runs the reference's own reference_tilemix (oracle/_ref)."""
    q, k, v = (_u16(_batched(t)) for t in (q, k, v))
    heads, m, d = q.shape
    n = k.shape[1]
    q8 = np.ascontiguousarray(_batched(q8), dtype=np.int8)
    k8 = np.ascontiguousarray(_batched(k8), dtype=np.int8)
    qs = _u16(np.asarray(q_scales).reshape(heads, -1))
    ks = _u16(np.asarray(k_scales).reshape(heads, -1))
    r = np.ascontiguousarray(routes, dtype=np.uint8).reshape(heads, -1)
    hid = np.ascontiguousarray(head_ids, dtype=np.int32)
    rid = np.ascontiguousarray(row_ids, dtype=np.int32)
    out = np.empty((hid.size, rid.size, d), np.float64)
    if use_reference:
        rl = ref_lib()
        if rl is None:
            raise RuntimeError("reference oracle (oracle/_ref) is not built")
        rl.ref_tilemix_sampled(_ptr(q), _ptr(k), _ptr(v), _ptr(q8), _ptr(qs), _ptr(k8), _ptr(ks),
                               _ptr(r), m, n, d, float(score_scale), int(causal), _ptr(hid),
                               hid.size, _ptr(rid), rid.size, _ptr(out))
    else:
        lib().orc_tilemix_sampled(_ptr(q), _ptr(k), _ptr(v), _ptr(q8), _ptr(k8), _ptr(qs),
                                  _ptr(ks), _ptr(r), m, n, d, float(score_scale), int(causal),
                                  _ptr(hid), hid.size, _ptr(rid), rid.size, _ptr(out))
    return out


def dense_attention(q, k, v) -> np.ndarray:
    """fp64 dense attention, scale 1/sqrt(d) (reference_attention.h:12-52)."""
    q, k, v = (_u16(t) for t in (q, k, v))
    m, d = q.shape
    out = np.empty((m, d), np.float64)
    lib().orc_dense_attention(_ptr(q), _ptr(k), _ptr(v), m, k.shape[0], d, _ptr(out))
    return out


def routing_policy(q_scales, k_scales, heads: int, m: int, n: int, key_tiles_per_group: int,
                   max_product: float) -> np.ndarray:
    """Routing words of the scale-product policy (orc_routing_policy): bit 1
    (INT8) iff q_scale(tile) * max k_scale(group) <= max_product in fp32."""
    qs = _u16(np.asarray(q_scales).reshape(heads, -1))
    ks = _u16(np.asarray(k_scales).reshape(heads, -1))
    out = np.empty(heads * routing_word_count(m, n, key_tiles_per_group), np.uint64)
    lib().orc_routing_policy(_ptr(qs), _ptr(ks), heads, m, n, key_tiles_per_group, ctypes.c_float(max_product),
                             _ptr(out))
    return out


def max_threads() -> int:
    return int(lib().orc_max_threads())


def set_threads(n: int) -> None:
    """OpenMP threads of both CPU checkers' later parallel regions on the
    calling thread (the reference build's too, when present)."""
    lib().orc_set_threads(int(n))
    if ref_available():
        ref_lib().ref_set_threads(int(n))


# ---------------------------------------------- the reference's own functions
def ref_quantize(x: np.ndarray, block_rows: int):
    xb = _u16(x)
    rows, d = xb.shape
    values = np.empty((rows, d), np.int8)
    scales = np.empty(((rows - 1) // block_rows + 1,), np.uint16)
    ref_lib().ref_quantize(_ptr(xb), rows, d, block_rows, _ptr(values), _ptr(scales))
    return values, scales.view(np.float16)


def ref_tilemix(q, k, v, q8, q_scales, k8, k_scales, routes, score_scale: float) -> np.ndarray:
    q, k, v = (_u16(t) for t in (q, k, v))
    m, d = q.shape
    n = k.shape[0]
    out = np.empty((m, d), np.float64)
    ref_lib().ref_tilemix(_ptr(q), _ptr(k), _ptr(v), _ptr(np.ascontiguousarray(q8)),
                          _ptr(_u16(q_scales)), _ptr(np.ascontiguousarray(k8)),
                          _ptr(_u16(k_scales)), _ptr(np.ascontiguousarray(routes, np.uint8)),
                          m, n, d, float(score_scale), _ptr(out))
    return out


def ref_attention(q, k, v) -> np.ndarray:
    q, k, v = (_u16(t) for t in (q, k, v))
    m, d = q.shape
    out = np.empty((m, d), np.float64)
    ref_lib().ref_attention(_ptr(q), _ptr(k), _ptr(v), m, k.shape[0], d, _ptr(out))
    return out


def ref_int8_dot(q8, k8, query: int, key: int) -> int:
    m, d = q8.shape
    return int(ref_lib().ref_int8_dot(_ptr(np.ascontiguousarray(q8)), _ptr(np.ascontiguousarray(k8)),
                                      m, k8.shape[0], query, key, d))


def threads_env() -> int:
    return int(os.environ.get("OMP_NUM_THREADS", "0") or 0) or max_threads()
