"""ctypes binding of libdsa_b200.so (the C ABI declared in include/dsa_b200.h).

The library is built in-tree by flashinfer_repo_b200.build.  There is no
fallback: if the library is missing or a call fails, an exception is raised.
"""
from __future__ import annotations

import ctypes
import os

from . import build as _build

_lib = None

I64 = ctypes.c_int64
P = ctypes.c_void_p
SZ = ctypes.c_size_t
F32 = ctypes.c_float
INT = ctypes.c_int

class Options(ctypes.Structure):
    """struct dsa_options (include/dsa_b200.h)."""
    _fields_ = [("attention_kernel", ctypes.c_int), ("attention_stages", ctypes.c_int),
                ("attention_ctas", ctypes.c_int), ("attention_min_tiles", ctypes.c_int),
                ("attention_grids", ctypes.c_int), ("merge_pdl", ctypes.c_int),
                ("indexer_tiles_per_cta", ctypes.c_int), ("attention_cluster", ctypes.c_int)]


# name -> argtypes; every function returns int (dsa_status) except the message.
SIGNATURES = {
    "dsa_sparse_attention_workspace_size": [I64, I64, I64, ctypes.POINTER(SZ)],
    "dsa_set_options": [ctypes.POINTER(Options)],
    "dsa_get_options": [ctypes.POINTER(Options)],
    "dsa_sparse_attention": [P, I64, I64, P, I64, I64, P, I64, I64, P, I64, I64, P, I64,
                             I64, I64, I64, I64, I64, F32, P, I64, I64, P, I64, I64, P, SZ, P],
    "dsa_sparse_attention_noalloc": [P, I64, I64, P, I64, I64, P, I64, I64, P, I64, I64, P, I64,
                                     I64, I64, I64, I64, I64, F32, P, I64, I64, P, I64, I64, P],
    "dsa_sparse_attention_noalloc_read_error": [INT, ctypes.POINTER(INT), P],
    "dsa_sparse_attention_scatter": [P, I64, I64, P, I64, I64, P, I64, I64, P, I64, I64, P, I64,
                                     I64, I64, I64, I64, I64, F32, P, I64, I64, P, I64, I64, INT,
                                     P, SZ, P],
    "dsa_sparse_attention_scatter_sync": [P, I64, I64, P, I64, I64, P, I64, I64, P, I64, I64, P, I64,
                                          I64, I64, I64, I64, I64, F32, P, I64, I64, P, I64, I64,
                                          INT, P, INT, INT, P, SZ, P],
    "dsa_peer_alloc": [SZ, ctypes.POINTER(P), P],
    "dsa_peer_open": [P, ctypes.POINTER(P)],
    "dsa_peer_close": [P],
    "dsa_peer_free": [P],
    "dsa_peer_barrier": [P, INT, INT, P, P],
    "dsa_read_device_error": [P, INT, ctypes.POINTER(INT), P],
    "dsa_indexer_scores": [P, P, I64, P, I64, P, P, I64, P, I64, I64, I64, I64, I64, P, I64, P, P],
    "dsa_index_cache_append": [P, I64, P, P, I64, P, I64, I64, P, P],
    "dsa_topk_select": [P, I64, P, P, I64, I64, I64, P, P, INT, P],
    "dsa_indexer_topk": [P, P, I64, P, I64, P, P, I64, P, I64, I64, I64, I64, I64, I64, P, P, P,
                         INT, P, P],
}


class DSAError(RuntimeError):
    """A failing call of the native library (status code + message)."""

    def __init__(self, fn, code, msg):
        super().__init__(f"{fn} failed with status {code}: {msg}")
        self.code = code


def lib_path() -> str:
    return _build.LIB


def load(build_if_missing: bool = True):
    global _lib
    if _lib is not None:
        return _lib
    path = lib_path()
    if not os.path.exists(path):
        if not build_if_missing:
            raise OSError(f"{path} is missing; run python -m flashinfer_repo_b200.build")
        _build.build()
    lib = ctypes.CDLL(path)
    lib.dsa_last_error_message.restype = ctypes.c_char_p
    lib.dsa_last_error_message.argtypes = []
    for name, args in SIGNATURES.items():
        f = getattr(lib, name)
        f.argtypes = args
        f.restype = INT
    _lib = lib
    return lib


def check(fn_name: str, rc: int):
    if rc != 0:
        msg = load().dsa_last_error_message().decode(errors="replace")
        raise DSAError(fn_name, rc, msg)


def call(fn_name: str, *args):
    check(fn_name, getattr(load(), fn_name)(*args))
