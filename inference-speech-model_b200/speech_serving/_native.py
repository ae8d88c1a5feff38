"""ctypes binding of libspd_b200.so, the C-ABI extension that holds every decode-path kernel.

This is the binding a Python caller of the C ABI (``include/spd_b200.h``) needs: it
loads the in-tree library, declares each exported function's argument types, and turns
non-zero status codes into ``RuntimeError`` with the library's own message (the
reference raises ``RuntimeError``/``ValueError`` for the same conditions, e.g.
speech_serving/block_manager.py:143-147, speech_serving/graph_decode_buffers.py:152-153).

There is no fallback: if the library is missing the import of an op fails loudly.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

_PKG_ROOT = Path(__file__).resolve().parent.parent
LIB_PATH = Path(os.environ.get("SPD_B200_LIB", _PKG_ROOT / "lib" / "libspd_b200.so"))

SPD_OK = 0
SPD_ERR_INVALID_ARG = 1
SPD_ERR_UNSUPPORTED = 2
SPD_ERR_CUDA = 3
SPD_ERR_WORKSPACE = 4

SPD_F32, SPD_F16, SPD_BF16 = 0, 1, 2

SPD_DEVERR_BLOCK_ID = 1
SPD_DEVERR_LENGTH = 2
SPD_DEVERR_TIMEOUT = 4

SPD_ACT_NONE, SPD_ACT_GELU = 0, 1

# Every symbol the header declares, with (restype, argtypes).
_vp, _i, _i64, _f, _sz = C.c_void_p, C.c_int, C.c_int64, C.c_float, C.c_size_t
_SIGNATURES = {
    "spd_version": (_i, []),
    "spd_get_last_error": (_i, [C.c_char_p, _sz]),
    "spd_paged_decode_attn_workspace_size": (_sz, [_i, _i, _i, _i, _i]),
    "spd_cross_attn_workspace_size": (_sz, [_i, _i, _i, _i]),
    "spd_read_error_word": (_i, [_vp, C.POINTER(C.c_int32), _vp]),
    "spd_paged_decode_attn": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _f, _i,
                                   _vp, _vp, _vp, _sz, _vp]),
    "spd_cross_attn": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i64, _i64, _f, _i, _vp, _sz, _vp]),
    "spd_kv_append": (_i, [_vp, _vp, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i,
                           _vp, _vp]),
    "spd_block_gather": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i64, _i, _i, _vp, _vp]),
    "spd_cross_kv_project": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i64, _i, _vp, _vp]),
    "spd_add_layernorm": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i64, _f, _i, _vp]),
    "spd_argmax_rows": (_i, [_vp, _i, _i, _i64, _vp, _vp, _i, _vp]),
    "spd_linear": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i64, _i64, _i, _i, _vp, _vp]),
    "spd_set_wait_timeout_ns": (_i, [C.c_uint64]),
    "spd_get_wait_timeout_ns": (C.c_uint64, []),
    "spd_selftest_wait_timeout": (_i, [_vp, C.c_uint64, _vp]),
    "spd_paged_decode_attn_noalloc": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _f, _i, _vp, _vp,
                                           _vp, _vp]),
}

_lib = None


def load() -> C.CDLL:
    """Loads the library once and declares every function signature."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(
            f"libspd_b200.so not found at {LIB_PATH}; build it with "
            "`python inference-speech-model_b200/csrc/build.py` (there is no CPU fallback)"
        )
    lib = C.CDLL(str(LIB_PATH))
    for name, (res, args) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)


def last_error() -> str:
    buf = C.create_string_buffer(512)
    load().spd_get_last_error(buf, 512)
    return buf.value.decode(errors="replace")


def check(rc: int, what: str) -> None:
    if rc != SPD_OK:
        raise RuntimeError(f"{what} failed (status {rc}): {last_error()}")
