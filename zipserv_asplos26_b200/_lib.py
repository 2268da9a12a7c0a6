"""ctypes binding of libzipserv_b200.so (the C ABI in include/zipserv_b200.h).

There is no fallback: if the library is missing or fails to load, every entry
point raises. Build it with `python -m zipserv_asplos26_b200.build_lib`.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

from .build_lib import LIB

_P = C.c_void_p
_I = C.c_int
_lock = threading.Lock()
_lib = None

_SIGS = {
    "zs_version": ([], _I),
    "zs_analyze_exponents_host": ([_P, C.c_int64, _I, _P], _I),
    "zs_encode_host": ([_P, _I, _I, _P] + [_P] * 9, _I),
    "zs_analyze_scratch_bytes": ([], C.c_size_t),
    "zs_analyze_exponents": ([_P, _P, C.c_int64, _I, _P, _P], _I),
    "zs_encode_scratch_bytes": ([_I, _I], C.c_size_t),
    "zs_encode": ([_P, _P, _I, _I, _P] + [_P] * 10, _I),
    "zs_decompress": ([_P] * 8 + [_I, _I, _I, _P, _I, _I, _P], _I),
    "zs_zipgemm": ([_P] * 8 + [_I, _I, _I, _P, _P, _I, _I, _I, _I, _P], _I),
    "zs_zipgemm_allreduce_buffer_bytes": ([_I, _I, _I], C.c_size_t),
    "zs_zipgemm_allreduce_counters": ([_I, _I], C.c_size_t),
    "zs_zipgemm_allreduce": ([_P] * 8 + [_I, _I, _I, _P, _P, _I, _I, _I, _I, _I, _P, _P, _P], _I),
    "zs_peer_handle_bytes": ([], C.c_size_t),
    "zs_peer_alloc": ([C.c_size_t, _P, _P], _I),
    "zs_peer_open": ([_P, _P], _I),
    "zs_peer_close": ([_P], _I),
    "zs_peer_free": ([_P], _I),
    "zs_decode_attention_workspace_bytes": ([_I, _I, _I, _I], C.c_size_t),
    "zs_decode_attention_default_splits": ([_I, _I, _I], _I),
    "zs_decode_attention_dense": ([_P, _P, _P, _P, _P] + [_I] * 6 + [C.c_float, _I, _P, C.c_size_t, _P, _P, _P], _I),
    "zs_decode_attention": ([_P, _P, _P, _P, _P, _P, _P] + [_I] * 6 + [C.c_float, _I, _P, C.c_size_t, _P, _P, _P],
                            _I),
}


class ZipServError(RuntimeError):
    pass


def lib():
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB):
                    raise ZipServError(f"{LIB} is not built (python -m zipserv_asplos26_b200.build_lib)")
                L = C.CDLL(LIB)
                for name, (args, res) in _SIGS.items():
                    fn = getattr(L, name)
                    fn.argtypes = args
                    fn.restype = res
                _lib = L
    return _lib


def exported_symbols():
    return list(_SIGS)


def check(status: int, what: str):
    if status != 0:
        raise ZipServError(f"{what} failed with cudaError {status}")
