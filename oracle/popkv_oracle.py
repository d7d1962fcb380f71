"""CPU oracle for the Pop-KV retrieval path -- TEST INFRASTRUCTURE ONLY.

numpy front end over ``popkv_oracle.c`` (the bit-exact restatement of the
reference kernel semantics).  Only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline leg import this module, as the checker; the shipped
library never does.

Reference anchors (kw78999/FIER-2bits):
  pack_keys      -> csrc/popkv_ext.cu:29-91   popkv_pack_g32_kernel
  pack_queries   -> csrc/popkv_ext.cu:117-149 (query pack inside popkv_score_kernel)
  score          -> csrc/popkv_ext.cu:150-177
  select         -> popkv.py:594-600 + _append_current popkv.py:141-145
  attention      -> popkv.py:341-368 gather_selected_kv + selected_attention
"""
from __future__ import annotations

import ctypes
import math
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "_build" / "libpopkv_oracle.so"
_lib = None


def build() -> Path:
    src = _HERE / "popkv_oracle.c"
    if not _LIB_PATH.exists() or _LIB_PATH.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)
    return _LIB_PATH


def _load():
    global _lib
    if _lib is None:
        build()
        lib = ctypes.CDLL(str(_LIB_PATH))
        P = ctypes.c_void_p
        I = ctypes.c_int64
        lib.oracle_pack_keys.argtypes = [P, I, I, I, I, I, I, P, P, P, P, P]
        lib.oracle_pack_queries.argtypes = [P, I, I, P, P, P, P]
        lib.oracle_score.argtypes = [P, I, I, I, P, P, P, P, I, I, ctypes.c_int, P, P,
                                     ctypes.c_float, P, I]
        lib.oracle_select.argtypes = [P, I, I, P, I, P]
        lib.oracle_attention.argtypes = [P, I, I, I, P, P, I, I, ctypes.c_int, P, P, P, P,
                                         I, P, P]
        for f in (lib.oracle_pack_keys, lib.oracle_pack_queries, lib.oracle_score,
                  lib.oracle_select, lib.oracle_attention):
            f.restype = None
        _lib = lib
    return _lib


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def default_scale(head_dim: int) -> float:
    """Correctly rounded fp32 1/sqrt(D), the scale the CUDA scorer uses."""
    return float(np.float32(1.0 / math.sqrt(head_dim)))


def pack_keys(keys, *, capacity: int | None = None, token_offset: int = 0,
              out=None, with_thresholds: bool = False):
    """keys [heads, T, D] (any float dtype, converted to float32 exactly).

    Returns (sign int32, mag int32, low uint16 fp16-bits, delta uint16) of shape
    [heads, capacity, words]; with ``with_thresholds`` also the
    [heads, groups, D, 2] fp32 (min*0.5, max*0.5) thresholds.
    """
    k = _f32(keys)
    heads, tokens, dim = k.shape
    words = (dim + 31) // 32
    cap = tokens + token_offset if capacity is None else int(capacity)
    if out is None:
        out = (np.zeros((heads, cap, words), np.int32), np.zeros((heads, cap, words), np.int32),
               np.zeros((heads, cap, words), np.uint16), np.zeros((heads, cap, words), np.uint16))
    groups = (tokens + 31) // 32
    thr = np.zeros((heads, groups, dim, 2), np.float32) if with_thresholds else None
    if tokens:
        _load().oracle_pack_keys(_ptr(k), heads, tokens, dim, tokens * dim, cap, token_offset,
                                 *(_ptr(x) for x in out), _ptr(thr))
    return (out, thr) if with_thresholds else out


def pack_queries(queries):
    q = _f32(queries)
    dim = q.shape[-1]
    rows = q.size // dim
    words = (dim + 31) // 32
    qs = np.zeros((rows, words), np.uint32)
    qm = np.zeros((rows, words), np.uint32)
    ql = np.zeros((rows, words), np.float32)
    qd = np.zeros((rows, words), np.float32)
    _load().oracle_pack_queries(_ptr(q), rows, dim, _ptr(qs), _ptr(qm), _ptr(ql), _ptr(qd))
    shape = q.shape[:-1] + (words,)
    return qs.reshape(shape), qm.reshape(shape), ql.reshape(shape), qd.reshape(shape)


def score(queries, packed, *, head_to_kv, tokens: int | None = None, lengths=None,
          kv_heads: int | None = None, cache_per_batch: bool = False, scale: float | None = None):
    """queries [B, QH, D]; packed 4-tuple [cache_heads, cap, W]. Returns fp32 [B, QH, tokens]."""
    q = _f32(queries)
    batch, q_heads, dim = q.shape
    sign, mag, low, delta = (np.ascontiguousarray(x) for x in packed)
    cap = sign.shape[1]
    h2k = np.ascontiguousarray(np.asarray(head_to_kv, dtype=np.int64))
    if lengths is None:
        lengths = np.full(batch, int(tokens), np.int64)
    lengths = np.ascontiguousarray(np.asarray(lengths, dtype=np.int64))
    width = int(tokens) if tokens is not None else int(lengths.max())
    kvh = sign.shape[0] if kv_heads is None else int(kv_heads)
    out = np.zeros((batch, q_heads, width), np.float32)
    _load().oracle_score(_ptr(q), batch, q_heads, dim, _ptr(sign), _ptr(mag), _ptr(low),
                         _ptr(delta), kvh, cap, int(cache_per_batch), _ptr(h2k), _ptr(lengths),
                         default_scale(dim) if scale is None else scale, _ptr(out), width)
    return out


def select(scores, *, budget: int, lengths=None):
    """scores [rows, >=L]; returns int32 [rows, budget] (sorted picks, newest, -1 pad)."""
    s = _f32(scores)
    s2 = s.reshape(-1, s.shape[-1])
    rows, stride = s2.shape
    if lengths is None:
        lengths = np.full(rows, stride, np.int64)
    lengths = np.ascontiguousarray(np.broadcast_to(np.asarray(lengths, np.int64), (rows,)))
    out = np.zeros((rows, budget), np.int32)
    _load().oracle_select(_ptr(s2), rows, stride, _ptr(lengths), budget, _ptr(out))
    return out


def attention(queries, key_cache, value_cache, *, head_to_kv, lengths, indices=None,
              budget: int | None = None, cur_keys=None, cur_values=None,
              cache_per_batch: bool = False, kv_heads: int | None = None):
    """Exact attention (fp64 accumulation). Shapes as in popkv_oracle.c."""
    q = _f32(queries)
    batch, q_heads, dim = q.shape
    kc, vc = _f32(key_cache), _f32(value_cache)
    kc = kc.reshape(-1, kc.shape[-2], dim)
    vc = vc.reshape(-1, vc.shape[-2], dim)
    kvh = (kc.shape[0] // batch if cache_per_batch else kc.shape[0]) if kv_heads is None else kv_heads
    h2k = np.ascontiguousarray(np.asarray(head_to_kv, dtype=np.int64))
    lengths = np.ascontiguousarray(np.broadcast_to(np.asarray(lengths, np.int64), (batch,)))
    idx = None
    if indices is not None:
        idx = np.ascontiguousarray(np.asarray(indices, np.int32).reshape(batch * q_heads, -1))
        budget = idx.shape[1]
    ck = None if cur_keys is None else _f32(cur_keys).reshape(batch, kvh, dim)
    cv = None if cur_values is None else _f32(cur_values).reshape(batch, kvh, dim)
    out = np.zeros((batch, q_heads, dim), np.float32)
    _load().oracle_attention(_ptr(q), batch, q_heads, dim, _ptr(kc), _ptr(vc), kvh, kc.shape[1],
                             int(cache_per_batch), _ptr(ck), _ptr(cv), _ptr(h2k), _ptr(idx),
                             int(budget or 0), _ptr(lengths), _ptr(out))
    return out


def f16_bits_to_float(bits: np.ndarray) -> np.ndarray:
    return np.asarray(bits, np.uint16).view(np.float16).astype(np.float32)
