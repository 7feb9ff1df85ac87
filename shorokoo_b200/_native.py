"""ctypes binding of include/shorokoo_b200.h (the library's C ABI)."""
from __future__ import annotations

import ctypes as C
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libshorokoo_b200.so")

_lib = None
_lock = threading.Lock()

P = C.c_void_p
I32, I64, SZ, DBL = C.c_int32, C.c_int64, C.c_size_t, C.c_double
CSTR = C.c_char_p
PSTR = C.POINTER(C.c_char_p)
PP = C.POINTER(C.c_void_p)

# name: (restype, argtypes)
SIGNATURES = {
    "sb_version": (I32, []),
    "sb_last_error": (CSTR, []),
    "sb_session_create": (I32, [C.c_char_p, SZ, I32, I32, PP]),
    "sb_session_create_ex": (I32, [C.c_char_p, SZ, I32, I32, I32, I32, I32, PP]),
    "sb_session_cache_clear": (I32, []),
    "sb_session_destroy": (None, [P]),
    "sb_session_input_count": (I32, [P]),
    "sb_session_input_name": (CSTR, [P, I32]),
    "sb_session_output_count": (I32, [P]),
    "sb_session_output_name": (CSTR, [P, I32]),
    "sb_session_run": (I32, [P, I32, PSTR, PP, I32, PSTR, PP]),
    "sb_session_run_device": (I32, [P, I32, PSTR, PP, I32, PSTR, PP]),
    "sb_value_device_ptr": (I32, [P, PP, C.POINTER(I32)]),
    "sb_value_create_tensor": (I32, [I32, C.POINTER(I64), I32, P, SZ, PP]),
    "sb_value_wrap_tensor": (I32, [I32, C.POINTER(I64), I32, P, SZ, PP]),
    "sb_value_create_string_tensor": (I32, [PSTR, SZ, C.POINTER(I64), I32, PP]),
    "sb_value_create_sequence": (I32, [PP, SZ, PP]),
    "sb_value_release": (None, [P]),
    "sb_value_type": (I32, [P]),
    "sb_value_elem_type": (I32, [P]),
    "sb_value_rank": (I32, [P]),
    "sb_value_shape": (C.POINTER(I64), [P]),
    "sb_value_data": (P, [P]),
    "sb_value_nbytes": (SZ, [P]),
    "sb_value_string_count": (SZ, [P]),
    "sb_value_string_at": (CSTR, [P, SZ]),
    "sb_value_count": (I32, [P]),
    "sb_value_at": (I32, [P, I32, PP]),
    "sb_value_sequence_elem_type": (I32, [P]),
    "sb_session_time_device": (I32, [P, I32, PSTR, PP, I32, I32, C.POINTER(DBL), I32, C.POINTER(I32)]),
    "sb_session_profile": (I32, [P, I32, PSTR, PP, I32, PSTR, C.POINTER(DBL), I32, C.POINTER(I32)]),
    "sb_session_stats": (I32, [P, I32, PSTR, PP, C.POINTER(I64), C.POINTER(I64), C.POINTER(DBL),
                               C.POINTER(I64), C.POINTER(I32)]),
    "sb_debug_lower": (I32, [C.c_char_p, SZ, I32, PP, C.c_char_p, SZ, C.POINTER(SZ)]),
    "sb_debug_narrow_bf16": (I32, [C.c_void_p, C.c_void_p, SZ, I32]),
    "sb_session_transfer_bytes": (I32, [P, I32, PSTR, PP, C.POINTER(I64), C.POINTER(I64)]),
    "sb_linear_noalloc": (I32, [P, P, P, P, I64, I64, I64, I32, P]),
}


def header_symbols() -> list:
    """Names declared in include/shorokoo_b200.h (parsed, so tests can compare with the .so)."""
    import re
    hdr = os.path.join(os.path.dirname(HERE), "include", "shorokoo_b200.h")
    with open(hdr) as f:
        return sorted(set(re.findall(r"\b(sb_[a-z0-9_]+)\s*\(", f.read())))


def lib():
    """Loads the library; raises (never falls back) if it is missing."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(f"{LIB_PATH} is missing; build it with `python -m shorokoo_b200.build`")
            l = C.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(l, name)
                fn.restype = res
                fn.argtypes = args
            _lib = l
        return _lib
