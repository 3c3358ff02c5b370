"""ctypes loader for ``libint4kv_b200.so`` (the C ABI in include/int4kv_b200.h).

The library is loaded from this package directory only (built in-tree by
``_build.py``); there is no fallback: if it is missing, every CUDA entry point
raises.
"""

import ctypes
import os

from ._build import LIB_PATH

_c_void_p = ctypes.c_void_p
_c_int = ctypes.c_int
_c_size_t = ctypes.c_size_t
_c_size_p = ctypes.POINTER(ctypes.c_size_t)

# name -> argtypes (every launcher returns cudaError_t as int)
_PROTOS = {
    "cu_quantize_int4": [_c_void_p, _c_int, _c_int, _c_void_p, _c_void_p, _c_void_p, _c_void_p],
    "cu_flash_decode_int4": [_c_void_p] * 6 + [_c_int] * 5 + [_c_void_p, _c_void_p],
    "int4kv_dense_decode_workspace_size": [_c_int] * 5 + [_c_size_p],
    "int4kv_dense_decode": [_c_void_p] * 6 + [_c_int] * 5 + [_c_void_p, _c_void_p, _c_size_t,
                                                              _c_void_p],
    "int4kv_quantize_grouped": [_c_void_p, _c_int, _c_int, _c_int, _c_int, _c_void_p, _c_void_p,
                                _c_void_p, _c_void_p],
    "int4kv_cache_write": [_c_void_p, _c_void_p, _c_void_p, _c_void_p] + [_c_int] * 6
                          + [_c_void_p, _c_int, _c_int] + [_c_void_p] * 5,
    "int4kv_paged_decode_workspace_size": [_c_int] * 4 + [_c_size_p],
    "int4kv_paged_decode": [_c_void_p] * 6 + [_c_int] * 8 + [_c_void_p, _c_void_p, _c_size_t,
                                                             _c_void_p, _c_void_p],
    "int4kv_paged_decode_profiled": [_c_void_p] * 6 + [_c_int] * 8
                                    + [_c_void_p, _c_void_p, _c_size_t] + [_c_void_p] * 4,
    "int4kv_paged_decode_workspace_size_ex": [_c_int] * 5 + [_c_size_p],
    "int4kv_paged_decode_ex": [_c_void_p, _c_void_p, _c_void_p, _c_int] + [_c_void_p] * 3
                              + [_c_int] * 8 + [_c_void_p, _c_void_p, _c_size_t] + [_c_void_p] * 4,
    "int4kv_cache_write_ex": [_c_void_p, _c_void_p, _c_void_p, _c_void_p] + [_c_int] * 6
                             + [_c_void_p, _c_int, _c_int] + [_c_void_p, _c_void_p, _c_int]
                             + [_c_void_p] * 3,
    "int4kv_stage_inputs": [_c_void_p, _c_void_p, _c_size_t, _c_void_p],
    "int4kv_cache_append": [_c_void_p] * 5 + [_c_int] * 6 + [_c_void_p, _c_int, _c_int]
                           + [_c_void_p, _c_void_p, _c_int] + [_c_void_p] * 3,
    "int4kv_rope": [_c_void_p, _c_void_p] + [_c_int] * 3 + [_c_void_p, _c_void_p, _c_int]
                   + [_c_void_p] * 3,
    "int4kv_cache_append_rope": [_c_void_p] * 5 + [_c_int] * 6 + [_c_void_p, _c_int, _c_int]
                                + [_c_void_p, _c_void_p, _c_int] + [_c_void_p] * 3 + [_c_int]
                                + [_c_void_p, _c_void_p, _c_int] + [_c_void_p, _c_void_p],
    "int4kv_block_decode": [_c_void_p] * 5 + [_c_int] + [_c_void_p] * 2 + [_c_int] * 6
                           + [_c_void_p, _c_void_p, _c_size_t, _c_void_p],
    "int4kv_paged_decode_partials": [_c_void_p] * 6 + [_c_int] * 8
                                    + [_c_void_p, _c_void_p, _c_size_t, _c_void_p, _c_void_p],
    "int4kv_paged_decode_partials_ex": [_c_void_p, _c_void_p, _c_void_p, _c_int] + [_c_void_p] * 3
                                       + [_c_int] * 8 + [_c_void_p, _c_void_p, _c_size_t,
                                                         _c_void_p, _c_void_p],
    "int4kv_merge_partials": [_c_void_p, _c_int, _c_int, _c_int, _c_void_p, _c_void_p],
    "int4kv_paged_decode_split_bytes": [_c_int, _c_int, _c_int, _c_size_p],
    "int4kv_paged_decode_split": [_c_void_p, _c_void_p, _c_void_p, _c_int] + [_c_void_p] * 3
                                 + [_c_int] * 8 + [_c_void_p, _c_int, _c_int]
                                 + [_c_void_p, _c_void_p, _c_size_t, _c_void_p, _c_void_p],
    "int4kv_exchange_bytes": [_c_int, _c_int, _c_int, _c_size_p],
    "int4kv_exchange_merge": [_c_void_p, _c_void_p] + [_c_int] * 4 + [_c_void_p] * 3,
    "int4kv_exchange_alloc": [_c_int, _c_size_t, ctypes.POINTER(_c_void_p)],
    "int4kv_exchange_free": [_c_void_p],
    "int4kv_ipc_handle": [_c_void_p, _c_void_p],
    "int4kv_ipc_open": [_c_void_p, ctypes.POINTER(_c_void_p)],
    "int4kv_ipc_close": [_c_void_p],
    "int4kv_paged_decode_static_scratch": [_c_void_p] * 6 + [_c_int] * 8
                                          + [_c_void_p, _c_void_p, _c_size_p, _c_void_p],
}

#: Every symbol include/int4kv_b200.h declares (checked by the CPU test suite).
EXPORTED = tuple(_PROTOS) + ("int4kv_build_info",)

_LIB = None


class LibraryMissing(RuntimeError):
    pass


def load():
    """Load the shared library once; raise LibraryMissing if it was never built."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not os.path.exists(LIB_PATH):
        raise LibraryMissing(
            f"{os.path.basename(LIB_PATH)} is not built; run __graft_entry__.build() "
            "(nvcc, sm_100a) first")
    lib = ctypes.CDLL(LIB_PATH)
    for name, argtypes in _PROTOS.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = ctypes.c_int
    lib.int4kv_build_info.argtypes = []
    lib.int4kv_build_info.restype = ctypes.c_char_p
    _LIB = lib
    return lib


def available():
    try:
        load()
        return True
    except (LibraryMissing, OSError):
        return False


def build_info():
    return load().int4kv_build_info().decode()


_ERRSTR = None


def error_string(code):
    """cudaGetErrorString through the CUDA runtime the library links."""
    global _ERRSTR
    if _ERRSTR is None:
        try:
            rt = ctypes.CDLL("libcudart.so.12")
        except OSError:
            rt = None
        if rt is not None:
            rt.cudaGetErrorString.argtypes = [ctypes.c_int]
            rt.cudaGetErrorString.restype = ctypes.c_char_p
            _ERRSTR = lambda c: rt.cudaGetErrorString(c).decode()  # noqa: E731
        else:
            _ERRSTR = lambda c: f"cudaError {c}"  # noqa: E731
    return _ERRSTR(code)


def check(code, what):
    if code != 0:
        raise RuntimeError(f"{what} failed: {error_string(code)} (cudaError {code})")
