"""ctypes binding of the C oracle (``plkv_oracle.c``).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).  The C file restates
the Rust CPU reference (crates/plkv-core/src/lib.rs); ``acc64=True`` runs the
same loops with FP64 accumulation.  ``build()`` compiles it with the
``Makefile`` beside it when the shared library is missing or stale.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
import threading

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "libplkv_oracle.so")
_SRC = os.path.join(_HERE, "plkv_oracle.c")
_LOCK = threading.Lock()
_LIB = None

_I64 = ctypes.c_int64
_P = ctypes.c_void_p
_F = ctypes.c_float
_INT = ctypes.c_int

STATUS_NAMES = {
    0: "ok", 1: "zero value", 2: "arithmetic overflow", 3: "invalid paged lookup",
    4: "token out of range", 5: "token not allocated", 6: "non-finite input",
    7: "fp16 overflow", 8: "invalid argument",
}


class OracleError(RuntimeError):
    def __init__(self, status: int, where: str):
        super().__init__(f"{where}: oracle status {status} ({STATUS_NAMES.get(status, '?')})")
        self.status = status


def build(force: bool = False) -> str:
    """Compile ``libplkv_oracle.so`` if it is missing or older than its source."""
    with _LOCK:
        stale = (not os.path.exists(_SO)) or os.path.getmtime(_SO) < os.path.getmtime(_SRC)
        if force or stale:
            subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _SO


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        build()
        L = ctypes.CDLL(_SO)
        sig = {
            "plkv_or_f32_to_f16_bits": (ctypes.c_uint16, [_F]),
            "plkv_or_f16_bits_to_f32": (_F, [ctypes.c_uint16]),
            "plkv_or_quantize_f16": (_INT, [_P, _I64, _P]),
            "plkv_or_resolve_location": (_INT, [_P, _I64, _I64, _I64, _I64, _P]),
            "plkv_or_latent_write_f16": (_INT, [_P, _I64, _I64, _I64, _P, _I64, _I64, _P]),
            "plkv_or_kv_write_f16": (_INT, [_P, _P, _I64, _I64, _I64, _I64, _P, _I64, _I64, _P, _P]),
            "plkv_or_project_query": (_INT, [_P, _P, _I64, _I64, _I64, _I64, _P]),
            "plkv_or_latent_decode_seq": (_INT, [_P, _P, _I64, _I64, _I64, _I64, _P, _I64, _I64,
                                                 _I64, _I64, _F, _P, _I64, _I64, _P, _P, _P, _P,
                                                 _I64, _I64, _INT]),
            "plkv_or_fullkv_decode_seq": (_INT, [_P, _P, _P, _I64, _I64, _I64, _I64, _P, _I64, _I64,
                                                 _I64, _I64, _F, _P, _P, _P, _I64, _I64, _INT]),
            "plkv_or_latent_decode_batch": (_INT, [_P, _P, _I64, _I64, _I64, _I64, _P, _I64, _P,
                                                   _I64, _I64, _F, _P, _I64, _I64, _P, _INT, _INT]),
            "plkv_or_fullkv_decode_batch": (_INT, [_P, _P, _P, _I64, _I64, _I64, _I64, _P, _I64, _P,
                                                   _I64, _I64, _F, _P, _INT, _INT]),
            "plkv_or_out_proj": (_INT, [_P, _P, _I64, _I64, _I64, _P, _INT, _INT]),
            "plkv_or_reconstruct_kv": (_INT, [_P, _I64, _I64, _I64, _P, _P, _I64, _P, _P, _INT]),
            "plkv_or_max_threads": (_INT, []),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = L
    return _LIB


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _c(a, dtype) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=dtype))


def _check(status: int, where: str) -> None:
    if status != 0:
        raise OracleError(status, where)


def f32_to_f16_bits(values) -> np.ndarray:
    """Element-wise RNE FP32 -> FP16 bits (no finiteness checks)."""
    L = lib()
    flat = _c(values, np.float32).ravel()
    out = np.fromiter((L.plkv_or_f32_to_f16_bits(float(x)) for x in flat), dtype=np.uint16,
                      count=flat.size)
    return out.reshape(np.shape(values))


def quantize_f16(values) -> np.ndarray:
    """lib.rs:302-319 -- FP16 storage bits; raises on non-finite / overflow."""
    v = _c(values, np.float32)
    out = np.empty(v.shape, dtype=np.uint16)
    _check(lib().plkv_or_quantize_f16(_ptr(v), v.size, _ptr(out)), "quantize_f16")
    return out


def resolve_location(table, pos: int, block_size: int, num_physical: int) -> tuple[int, int, int]:
    t = _c(table, np.int64)
    out = np.zeros(3, dtype=np.int64)
    _check(lib().plkv_or_resolve_location(_ptr(t), t.size, pos, block_size, num_physical,
                                          _ptr(out)), "resolve_location")
    return int(out[0]), int(out[1]), int(out[2])


def latent_write_f16(cache_bits: np.ndarray, table, pos: int, new_row) -> np.ndarray:
    """lib.rs:889-939 on a copy of ``cache_bits`` [P, bs, L] uint16."""
    cache = np.array(cache_bits, dtype=np.uint16, copy=True, order="C")
    t = _c(table, np.int64)
    row = _c(new_row, np.float32)
    P, bs, L = cache.shape
    _check(lib().plkv_or_latent_write_f16(_ptr(cache), P, bs, L, _ptr(t), t.size, pos, _ptr(row)),
           "latent_write_f16")
    return cache


def kv_write_f16(k_bits, v_bits, table, pos: int, new_k, new_v):
    """lib.rs:190-247 for FP16 head-major [P, KV, bs, D] storage, on copies."""
    k = np.array(k_bits, dtype=np.uint16, copy=True, order="C")
    v = np.array(v_bits, dtype=np.uint16, copy=True, order="C")
    t = _c(table, np.int64)
    nk = _c(new_k, np.float32)
    nv = _c(new_v, np.float32)
    P, KV, bs, D = k.shape
    _check(lib().plkv_or_kv_write_f16(_ptr(k), _ptr(v), P, KV, bs, D, _ptr(t), t.size, pos,
                                      _ptr(nk), _ptr(nv)), "kv_write_f16")
    return k, v


def project_query(q, w_k_canonical, kv_heads: int) -> np.ndarray:
    """lib.rs:1026-1032; ``q [Hq, D]``, ``w_k_canonical [L, KV*D]`` -> ``[Hq, L]``."""
    qq = _c(q, np.float32)
    w = _c(w_k_canonical, np.float32)
    Hq, D = qq.shape
    L = w.shape[0]
    out = np.empty((Hq, L), dtype=np.float32)
    _check(lib().plkv_or_project_query(_ptr(qq), _ptr(w), Hq, kv_heads, D, L, _ptr(out)),
           "project_query")
    return out


def latent_decode_seq(q_lat, cache_bits, table, active: int, max_len: int, block_size: int,
                      scale: float, value_dim: int | None = None, w_v_canonical=None,
                      proj_heads: int = 1, head_dim: int = 0, heads: tuple[int, int] | None = None,
                      acc64: bool = False, want_intermediates: bool = True):
    """lib.rs:941-1145 for one sequence.  Returns (scores, probs, ctx_lat, ctx)."""
    ql = _c(q_lat, np.float32)
    cache = np.ascontiguousarray(cache_bits, dtype=np.uint16)
    t = _c(table, np.int32)
    Hq, L = ql.shape
    P = cache.shape[0]
    Lv = L if value_dim is None else value_dim
    w = None if w_v_canonical is None else _c(w_v_canonical, np.float32)
    scores = np.zeros((Hq, max_len), np.float32) if want_intermediates else None
    probs = np.zeros((Hq, max_len), np.float32) if want_intermediates else None
    ctx_lat = np.zeros((Hq, Lv), np.float32)
    ctx = np.zeros((Hq, head_dim), np.float32) if w is not None else None
    h0, h1 = heads if heads is not None else (0, Hq)
    _check(lib().plkv_or_latent_decode_seq(
        _ptr(ql), _ptr(cache), P, block_size, L, Lv, _ptr(t), t.size, active, max_len, Hq,
        scale, _ptr(w), proj_heads, head_dim, _ptr(scores), _ptr(probs), _ptr(ctx_lat), _ptr(ctx),
        h0, h1, int(acc64)), "latent_decode_seq")
    return scores, probs, ctx_lat, ctx


def fullkv_decode_seq(q, k_bits, v_bits, table, active: int, max_len: int, scale: float,
                      heads: tuple[int, int] | None = None, acc64: bool = False):
    """lib.rs:1147-1269 for one sequence; K/V head-major [P, KV, bs, D] uint16."""
    qq = _c(q, np.float32)
    k = np.ascontiguousarray(k_bits, dtype=np.uint16)
    v = np.ascontiguousarray(v_bits, dtype=np.uint16)
    t = _c(table, np.int32)
    Hq, D = qq.shape
    P, KV, bs, _ = k.shape
    scores = np.zeros((Hq, max_len), np.float32)
    probs = np.zeros((Hq, max_len), np.float32)
    ctx = np.zeros((Hq, D), np.float32)
    h0, h1 = heads if heads is not None else (0, Hq)
    _check(lib().plkv_or_fullkv_decode_seq(
        _ptr(qq), _ptr(k), _ptr(v), P, KV, bs, D, _ptr(t), t.size, active, max_len, Hq, scale,
        _ptr(scores), _ptr(probs), _ptr(ctx), h0, h1, int(acc64)), "fullkv_decode_seq")
    return scores, probs, ctx


def latent_decode_batch(q_lat, cache_bits, tables, lens, block_size: int, scale: float,
                        value_dim: int, w_v_canonical, proj_heads: int, head_dim: int,
                        acc64: bool = False, threads: int = 0) -> np.ndarray:
    """Batched per-sequence-table latent decode -> ctx [B, Hq, D] (OpenMP)."""
    ql = _c(q_lat, np.float32)
    cache = np.ascontiguousarray(cache_bits, dtype=np.uint16)
    tb = _c(tables, np.int32)
    ln = _c(lens, np.int32)
    w = _c(w_v_canonical, np.float32)
    B, Hq, L = ql.shape
    ctx = np.zeros((B, Hq, head_dim), np.float32)
    _check(lib().plkv_or_latent_decode_batch(
        _ptr(ql), _ptr(cache), cache.shape[0], block_size, L, value_dim, _ptr(tb), tb.shape[1],
        _ptr(ln), B, Hq, scale, _ptr(w), proj_heads, head_dim, _ptr(ctx), int(acc64), threads),
        "latent_decode_batch")
    return ctx


def fullkv_decode_batch(q, k_bits, v_bits, tables, lens, scale: float, acc64: bool = False,
                        threads: int = 0) -> np.ndarray:
    """Batched per-sequence-table full-KV decode -> ctx [B, Hq, D] (OpenMP)."""
    qq = _c(q, np.float32)
    k = np.ascontiguousarray(k_bits, dtype=np.uint16)
    v = np.ascontiguousarray(v_bits, dtype=np.uint16)
    tb = _c(tables, np.int32)
    ln = _c(lens, np.int32)
    B, Hq, D = qq.shape
    P, KV, bs, _ = k.shape
    ctx = np.zeros((B, Hq, D), np.float32)
    _check(lib().plkv_or_fullkv_decode_batch(
        _ptr(qq), _ptr(k), _ptr(v), P, KV, bs, D, _ptr(tb), tb.shape[1], _ptr(ln), B, Hq, scale,
        _ptr(ctx), int(acc64), threads), "fullkv_decode_batch")
    return ctx


def out_proj(x, w, acc64: bool = False, threads: int = 0) -> np.ndarray:
    xx = _c(x, np.float32)
    ww = _c(w, np.float32)
    B, K = xx.shape
    N = ww.shape[1]
    out = np.zeros((B, N), np.float32)
    _check(lib().plkv_or_out_proj(_ptr(xx), _ptr(ww), B, K, N, _ptr(out), int(acc64), threads),
           "out_proj")
    return out


def reconstruct_kv(latent, w_k, w_v, acc64: bool = False) -> tuple[np.ndarray, np.ndarray]:
    """lib.rs:517-580: token-major K, V [T, width] from latent rows [T, L],
    w_k [L, width], w_v [Lv, width] (canonical)."""
    lat = _c(latent, np.float32)
    wk = _c(w_k, np.float32)
    wv = _c(w_v, np.float32)
    T, L = lat.shape
    W = wk.shape[1]
    k = np.zeros((T, W), np.float32)
    v = np.zeros((T, W), np.float32)
    _check(lib().plkv_or_reconstruct_kv(_ptr(lat), T, L, wv.shape[0], _ptr(wk), _ptr(wv), W,
                                        _ptr(k), _ptr(v), int(acc64)), "reconstruct_kv")
    return k, v


def max_threads() -> int:
    return int(lib().plkv_or_max_threads())
