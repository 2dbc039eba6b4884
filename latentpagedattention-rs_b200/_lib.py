"""ctypes binding of libplkv_b200.so (the C ABI declared in include/plkv_b200.h).

There is no fallback: if the shared library is missing the import of the
operations fails with an error that says how to build it.
"""

from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libplkv_b200.so")

_I32 = ctypes.c_int32
_I64 = ctypes.c_int64
_P = ctypes.c_void_p
_F = ctypes.c_float
_SZ = ctypes.c_size_t

PLKV_OK = 0
PLKV_ERR_ZERO_VALUE = 1
PLKV_ERR_ARITHMETIC_OVERFLOW = 2
PLKV_ERR_INVALID_PAGED_LOOKUP = 3
PLKV_ERR_TOKEN_OUT_OF_RANGE = 4
PLKV_ERR_TOKEN_NOT_ALLOCATED = 5
PLKV_ERR_NON_FINITE = 6
PLKV_ERR_FP16_OVERFLOW = 7
PLKV_ERR_INVALID_ARGUMENT = 8
PLKV_ERR_WORKSPACE = 9
PLKV_ERR_CUDA = 10
PLKV_ERR_UNSUPPORTED = 11

FLAG_NON_FINITE_INPUT = 0x1
FLAG_FP16_OVERFLOW = 0x2
FLAG_BAD_BLOCK = 0x4
FLAG_BAD_POSITION = 0x8
FLAG_BAD_LENGTH = 0x10
FLAG_TIMEOUT = 0x20

MODE_EXACT_F32 = 0
MODE_TC_F16 = 1


class WorkItem(ctypes.Structure):
    _fields_ = [("seq", _I32), ("block_begin", _I32), ("block_end", _I32), ("reserved", _I32)]


class LatentDecodeArgs(ctypes.Structure):
    _fields_ = [
        ("q_lat", _P), ("cache", _P), ("num_physical", _I64), ("block_size", _I32),
        ("latent_dim", _I32), ("value_dim", _I32), ("batch", _I32), ("q_heads", _I32),
        ("scale", _F), ("block_tables", _P), ("max_blocks", _I64), ("seq_lens", _P),
        ("items", _P), ("seq_item_begin", _P), ("n_items", _I32),
        ("worker_item_begin", _P), ("n_workers", _I32), ("allow_empty", _I32), ("w_v", _P), ("proj_heads", _I32), ("head_dim", _I32), ("ctx", _P), ("lse", _P),
        ("scores", _P), ("probs", _P), ("max_seq_len", _I32), ("mode", _I32),
        ("workspace", _P), ("workspace_bytes", _SZ), ("err_flags", _P),
    ]


class FullKVDecodeArgs(ctypes.Structure):
    _fields_ = [
        ("q", _P), ("k_cache", _P), ("v_cache", _P), ("num_physical", _I64), ("kv_heads", _I32),
        ("block_size", _I32), ("head_dim", _I32), ("batch", _I32), ("q_heads", _I32),
        ("scale", _F), ("block_tables", _P), ("max_blocks", _I64), ("seq_lens", _P),
        ("items", _P), ("seq_item_begin", _P), ("n_items", _I32), ("allow_empty", _I32),
        ("ctx", _P), ("lse", _P), ("scores", _P), ("probs", _P), ("max_seq_len", _I32),
        ("workspace", _P), ("workspace_bytes", _SZ), ("err_flags", _P),
    ]


# Every symbol of include/plkv_b200.h with its (restype, argtypes).
SIGNATURES = {
    "plkv_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "plkv_version": (ctypes.c_int, []),
    "plkv_quantize_f16": (ctypes.c_int, [_P, _P, _I64, _P, _P]),
    "plkv_latent_append_f16": (ctypes.c_int, [_P, _P, _I64, _P, _P, _P, _I64, _P, _I64, _I32,
                                              _I32, _P, _P]),
    "plkv_latent_append_slots_f16": (ctypes.c_int, [_P, _P, _I64, _P, _I64, _I32, _P, _P]),
    "plkv_reconstruct_kv": (ctypes.c_int, [_P, _I32, _I64, _I32, _I32, _P, _I64, _P, _P, _I32,
                                            _I32, _I32, _P, _P, _I32, _P, _P]),
    "plkv_peer_buffer_bytes": (_SZ, [_I64, _I32]),
    "plkv_peer_alloc": (ctypes.c_int, [_SZ, _P, _P]),
    "plkv_peer_init_buffer": (ctypes.c_int, [_P, _SZ, _P]),
    "plkv_peer_open": (ctypes.c_int, [_P, _P]),
    "plkv_peer_close": (ctypes.c_int, [_P]),
    "plkv_peer_free": (ctypes.c_int, [_P]),
    "plkv_peer_publish": (ctypes.c_int, [_P, _P, _I64, _I32, _P, _I32, _I32, _P, _P, _P]),
    "plkv_peer_merge": (ctypes.c_int, [_I64, _I32, _P, _I32, _I32, _P, _P, _P, _P, _P]),
    "plkv_allocate_slots": (ctypes.c_int, [_P, _I64, _P, _P, _I32, _I32, _P, _I64, _P, _I64, _P,
                                            _P]),
    "plkv_kv_append_f16": (ctypes.c_int, [_P, _P, _P, _I64, _P, _P, _P, _I64, _P, _P, _I64, _I32,
                                          _I32, _I32, _P, _P]),
    "plkv_plan_splits": (ctypes.c_int, [_P, _I32, _I32, _I32, _I32, _P, _I32, _P, _P]),
    "plkv_plan_workers": (ctypes.c_int, [_P, _I32, _I32, _I32, _P, _I32, _P, _P, _P]),
    "plkv_project_query": (ctypes.c_int, [_P, _P, _P, _I32, _I32, _I32, _I32, _I32, _P]),
    "plkv_latent_decode_workspace_size": (_SZ, [_I32, _I32, _I32, _I32, _I32]),
    "plkv_latent_decode": (ctypes.c_int, [ctypes.POINTER(LatentDecodeArgs), _P]),
    "plkv_latent_decode_partial": (ctypes.c_int, [ctypes.POINTER(LatentDecodeArgs), _P]),
    "plkv_latent_decode_combine": (ctypes.c_int, [ctypes.POINTER(LatentDecodeArgs), _P]),
    "plkv_latent_decode_noalloc": (ctypes.c_int, [ctypes.POINTER(LatentDecodeArgs), _P]),
    "plkv_lse_merge": (ctypes.c_int, [_P, _P, _I32, _I64, _I32, _P, _P, _P]),
    "plkv_out_proj_workspace_size": (_SZ, [_I32, _I32, _I32]),
    "plkv_out_proj": (ctypes.c_int, [_P, _P, _P, _I32, _I32, _I32, _I32, _P, _SZ, _P]),
    "plkv_out_proj_tc_workspace_size": (_SZ, [_I32, _I32, _I32]),
    "plkv_out_proj_tc": (ctypes.c_int, [_P, _P, _P, _I32, _I32, _I32, _I32, _P, _SZ, _P, _P]),
    "plkv_fullkv_decode_workspace_size": (_SZ, [_I32, _I32, _I32, _I32]),
    "plkv_fullkv_decode": (ctypes.c_int, [ctypes.POINTER(FullKVDecodeArgs), _P]),
    "plkv_selftest_bounded_wait": (ctypes.c_int, [_P, _P, _P, _P]),
    "plkv_shard_buffer_bytes": (_SZ, [_I32, _I32, _I32]),
    "plkv_shard_publish": (ctypes.c_int, [ctypes.POINTER(LatentDecodeArgs), _P, _I32, _I32, _P,
                                          _P]),
    "plkv_shard_merge": (ctypes.c_int, [_P, _I32, _I32, _P, _I32, _I32, _I32, _P, _I32, _P, _P,
                                        _P, _P]),
}

_LIB: ctypes.CDLL | None = None


class PlkvError(RuntimeError):
    """A non-zero plkv_status from the C ABI."""

    def __init__(self, status: int, where: str):
        msg = lib().plkv_status_string(status).decode() if _LIB is not None else str(status)
        super().__init__(f"{where}: {msg} (status {status})")
        self.status = status


def lib() -> ctypes.CDLL:
    """Load libplkv_b200.so once; raise if it has not been built."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build the CUDA library first "
                "(python latentpagedattention-rs_b200/build.py or __graft_entry__.build())")
        handle = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = handle
    return _LIB


def check(status: int, where: str) -> None:
    if status != PLKV_OK:
        raise PlkvError(status, where)
