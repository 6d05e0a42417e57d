"""ctypes binding of the C ABI in ``include/llmik.h`` (libllmik_b200.so).

This is the binding a non-PyTorch host (or a test) uses to call the library
directly with raw device pointers: every function takes plain integers and
pointers and returns a ``lik_status``; :func:`check` turns a non-zero status
into ``LikError`` carrying ``lik_last_error()``.
"""
from __future__ import annotations

import ctypes as C
import os

_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libllmik_b200.so")

LIK_OK = 0
STATUS_NAMES = {
    0: "LIK_OK", 1: "LIK_ERR_INVALID_ARGUMENT", 2: "LIK_ERR_UNSUPPORTED", 3: "LIK_ERR_MISALIGNED",
    4: "LIK_ERR_WORKSPACE", 5: "LIK_ERR_CUDA", 6: "LIK_ERR_DEVICE_TIMEOUT", 7: "LIK_ERR_DEVICE_BAD_BLOCK",
}

_p, _i64, _sz, _f, _int = C.c_void_p, C.c_int64, C.c_size_t, C.c_float, C.c_int

# name -> (restype, argtypes); must list every function of include/llmik.h
SIGNATURES = {
    "lik_abi_version": (_int, []),
    "lik_status_string": (C.c_char_p, [_int]),
    "lik_last_error": (C.c_char_p, []),
    "lik_decode_workspace_bytes": (_sz, [_i64, _i64, _i64]),
    "lik_workspace_init": (_int, [_p, _sz, _p]),
    "lik_workspace_check": (_int, [_p, _sz, _p, C.POINTER(_int)]),
    "lik_selftest_bounded_wait": (_int, [_i64, C.POINTER(_int), _p]),
    "lik_selftest_leave_timeout": (_int, [_i64, _p, _sz, _p]),
    "lik_decode_noalloc_check": (_int, [_p, C.POINTER(_int)]),
    "lik_decode_attention_f16": (_int, [_p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _f, _p, _sz, _p]),
    "lik_decode_attention_f16_noalloc": (_int, [_p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _f, _p]),
    "lik_decode_attention_int8": (_int, [_p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _f,
                                         _p, _sz, _p]),
    "lik_decode_attention_int4": (_int, [_p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                                         _i64, _f, _p, _sz, _p]),
    "lik_decode_attention_int4_asym": (_int, [_p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64,
                                              _i64, _i64, _i64, _f, _p, _sz, _p]),
    "lik_quantize_per_token_int8": (_int, [_p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _p]),
    "lik_quantize_v_per_token_int4": (_int, [_p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _p]),
    "lik_quantize_k_per_channel_groupwise_int4": (_int, [_p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                                                         _i64, _p]),
    "lik_quantize_v_per_token_int4_asym": (_int, [_p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _p]),
    "lik_quantize_k_per_channel_groupwise_int4_asym": (_int, [_p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64,
                                                              _i64, _i64, _i64, _p]),
    "lik_decode_attention_paged": (_int, [_int, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64,
                                          _i64, _i64, _i64, _i64, _i64, _f, _p, _sz, _p]),
    "lik_paged_append": (_int, [_int, _p, _p, _i64, _i64, _i64, _p, _p, _p, _i64, _i64, _p]),
    "lik_dequantize_int8": (_int, [_p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _p]),
    "lik_dequantize_int4": (_int, [_p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _p]),
    "lik_dequantize_int4_asym": (_int, [_p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                                        _p]),
}


class LikError(RuntimeError):
    def __init__(self, status: int, detail: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {detail}")
        self.status = status


_lib = None


def lib(path: str | None = None) -> C.CDLL:
    """Load libllmik_b200.so once and attach the signatures."""
    global _lib
    if _lib is None or path is not None:
        handle = C.CDLL(path or _LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def check(status: int) -> None:
    if status != LIK_OK:
        raise LikError(status, lib().lik_last_error().decode())


def call(name: str, *args) -> None:
    """Call an entry point returning lik_status and raise on failure."""
    check(getattr(lib(), name)(*args))
