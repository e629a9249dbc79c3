"""ctypes binding of libnvattn.so (the C ABI declared in include/nvattn.h).

This module is the only place that touches the shared library. It loads the
in-tree ``libnvattn.so`` (built by ``nvattn.build``), declares every entry
point's signature, and turns a non-zero return code into a Python exception
carrying ``nvattn_last_error()``. There is no fallback: if the library is
missing, importing anything that needs it raises.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import c_char_p, c_float, c_int, c_int32, c_int64, c_size_t, c_uint64, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libnvattn.so"

OK = 0
ERR_INVALID = 1
ERR_UNSUPPORTED = 2
ERR_CUDA = 3
ERR_WORKSPACE = 4

STATUS_BAD_SLOT = 1
STATUS_BAD_BLOCK = 2
STATUS_TIMEOUT = 4
STATUS_BAD_POSITION = 8

_P = c_void_p
_I32P = c_void_p

# name -> (restype, argtypes); mirrors include/nvattn.h
SIGNATURES: dict[str, tuple] = {
    "nvattn_last_error": (c_char_p, []),
    "nvattn_version": (c_int, []),
    "nvattn_store_kvcache": (c_int, [_P, c_int64, _P, c_int64, _P, _P, _I32P, c_int64, c_int64,
                                     c_int64, _I32P, _P]),
    "nvattn_varlen_prefill": (c_int, [_P, c_int64, c_int64,   # q
                                      _P, c_int64, c_int64,   # k
                                      _P, c_int64, c_int64,   # v
                                      _P, c_int64, c_int64,   # out
                                      _I32P, _I32P,           # cu_seqlens_q/k
                                      c_int32, c_int32, c_int32, c_int64, c_int64,
                                      _I32P, c_int64, c_int32, c_int32, c_int32,
                                      c_int32, c_int32, c_int32,
                                      c_float, c_int32, _I32P, _P]),
    "nvattn_decode_workspace_bytes": (c_size_t, [c_int32, c_int32, c_int32, c_int32, c_int32]),
    "nvattn_paged_decode": (c_int, [_P, c_int64, c_int64,    # q
                                    _P, _P,                  # caches
                                    _P, c_int64, c_int64,    # out
                                    _I32P, _I32P, c_int64,   # seqlens, block_table, stride
                                    c_int32, c_int32, c_int32,
                                    c_int32, c_int32, c_int32, c_int32,
                                    c_float, _P, c_size_t, _I32P, _P]),
    "nvattn_paged_decode_noalloc": (c_int, [_P, c_int64, c_int64, _P, _P, _P, c_int64, c_int64,
                                            _I32P, _I32P, c_int64, c_int32, c_int32, c_int32,
                                            c_int32, c_int32, c_int32, c_int32, c_float, _I32P,
                                            _P]),
    "nvattn_tree_workspace_bytes": (c_size_t, [c_int32, c_int32, c_int64, c_int32, c_int32,
                                               c_int32, c_int32]),
    "nvattn_tree_verify": (c_int, [_P, c_int64, c_int64,
                                   _P, _P,
                                   _P, c_int64, c_int64,
                                   _I32P, _I32P, _P,
                                   _I32P, c_int64, c_int32, c_int32, c_int32,
                                   c_int32, c_int32, c_int64,
                                   c_int32, c_int32, c_int32,
                                   c_float, _P, c_size_t, _I32P, _P]),
    "nvattn_kv_move": (c_int, [_P, _P, _I32P, _I32P, _I32P, c_int32, c_int32, c_int64, c_int64,
                               _I32P, _P]),
    "nvattn_qk_norm_rope_store": (c_int, [_P, c_int64, _P, c_int64, _P, c_int64,  # q, k, v
                                          _P, _P, _P, c_int64,   # weights, cos_sin, max_position
                                          _P, _I32P,             # positions, slot_mapping
                                          _P, _P, _P, _P,        # q_out, k_out, k/v caches
                                          c_int64, c_int64, c_int32, c_int32, c_int32,
                                          c_float, _I32P, _P]),
    "nvattn_sample": (c_int, [_P, c_int64, c_int64, c_int64, _P, c_uint64, c_uint64, _P, _P]),
    "nvattn_sample_shard": (c_int, [_P, c_int64, c_int64, c_int64, c_int64, _P, c_uint64, c_uint64,
                                    _P, _P]),
    "nvattn_sample_merge": (c_int, [_P, c_int64, c_int64, _P, _P]),
    "nvattn_ar_buffer_bytes": (c_size_t, [c_int64]),
    "nvattn_ar_alloc": (c_int, [c_size_t, _P, _P]),
    "nvattn_ar_open": (c_int, [_P, _P]),
    "nvattn_ar_close": (c_int, [_P]),
    "nvattn_ar_free": (c_int, [_P]),
    "nvattn_allreduce": (c_int, [_P, c_int32, c_int32, c_int64, c_int64, _P, _P, _I32P, _P]),
    "nvattn_ar_set_wait_limit": (c_int64, [c_int64]),
    "nvattn_ar_protocol": (c_int32, [c_int32, c_int64, c_int64]),
    "nvattn_decode_prepare_bytes": (c_size_t, [c_int64, c_int32]),
    "nvattn_decode_prepare": (c_int, [_P, _P, c_int64, c_int32, c_int32, c_int64,
                                      _P, _P, _I32P, _I32P, _I32P, c_int64, _I32P, _P]),
}


class NvattnError(RuntimeError):
    """A libnvattn entry point returned an error code."""

    def __init__(self, fn: str, code: int, msg: str):
        super().__init__(f"{fn} failed (code {code}): {msg}")
        self.code = code


_lib: ctypes.CDLL | None = None


def load(path: os.PathLike | str | None = None) -> ctypes.CDLL:
    """Load libnvattn.so once and declare all signatures."""
    global _lib
    if _lib is not None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise ImportError(
            f"{p} is missing: build the CUDA library first (python -m nvattn.build "
            "or __graft_entry__.build()); nvattn has no CPU fallback")
    lib = ctypes.CDLL(str(p))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def call(name: str, *args) -> int:
    """Call entry point `name`; raise NvattnError on a non-zero code."""
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != OK:
        msg = lib.nvattn_last_error().decode(errors="replace")
        raise NvattnError(name, rc, msg)
    return rc


def version() -> tuple[int, int]:
    v = load().nvattn_version()
    return v >> 16, v & 0xFFFF
