"""ctypes front end of the C oracle (oracle.c).  TEST INFRASTRUCTURE: imported only by
tests/ and by bench.py's CPU-baseline leg."""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from . import build_oracle

_lib = None
_DT = {np.dtype(np.float32): 0, np.dtype(np.float16): 1}


def _load():
    global _lib
    if _lib is None:
        try:
            _lib = C.CDLL(str(build_oracle.LIB))
        except OSError:
            _lib = C.CDLL(str(build_oracle.build(force=True)))
        vp, i, f, ll = C.c_void_p, C.c_int, C.c_float, C.c_longlong
        _lib.oracle_paged_attn.argtypes = [vp, vp, vp, vp, vp, vp, i, i, i, i, i, f, i, i]
        _lib.oracle_cross_attn.argtypes = [vp, vp, vp, vp, vp, i, i, i, i, ll, ll, f, i, i]
    return _lib


def _dtype_code(a: np.ndarray, bf16: bool) -> int:
    if bf16:
        return 2  # uint16 array holding bfloat16 bit patterns
    return _DT[a.dtype]


def paged_decode_attention(q, k_pool, v_pool, block_tables, context_lens, scale, threads=None, bf16=False):
    B, H, D = q.shape
    out = np.zeros((B, H, D), np.float32)
    tables = np.ascontiguousarray(block_tables, dtype=np.int32)
    ctx = np.ascontiguousarray(context_lens, dtype=np.int32)
    q, k_pool, v_pool = (np.ascontiguousarray(a) for a in (q, k_pool, v_pool))
    _load().oracle_paged_attn(q.ctypes.data, k_pool.ctypes.data, v_pool.ctypes.data, tables.ctypes.data,
                              ctx.ctypes.data, out.ctypes.data, B, H, D, k_pool.shape[1], tables.shape[1],
                              float(scale), _dtype_code(q, bf16), threads or os.cpu_count())
    return out


def cross_attention(q, k, v, valid_lens, scale, threads=None, bf16=False):
    B, H, D = q.shape
    T = k.shape[2]
    out = np.zeros((B, H, D), np.float32)
    valid = np.ascontiguousarray(valid_lens, dtype=np.int32)
    q, k, v = (np.ascontiguousarray(a) for a in (q, k, v))
    _load().oracle_cross_attn(q.ctypes.data, k.ctypes.data, v.ctypes.data, valid.ctypes.data, out.ctypes.data,
                              B, H, D, T, H * T * D, T * D, float(scale), _dtype_code(q, bf16),
                              threads or os.cpu_count())
    return out
