"""ctypes binding of libppmoe.so (the C ABI declared in include/ppmoe.h).

The shared library is built in-tree (``csrc/Makefile`` -> ``libppmoe.so`` beside this file).
There is no fallback: if the library is missing or fails to load, importing the modules
that need it raises immediately.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libppmoe.so")

ERR = {0: "ok", -1: "invalid argument", -2: "unsupported shape", -3: "device wait timed out",
       -4: "CUDA error", -5: "workspace"}

DECODE_MAX_TOKENS = 16

_c_void_p = ctypes.c_void_p
_c_int = ctypes.c_int
_c_size_t = ctypes.c_size_t
_c_float = ctypes.c_float

# name -> (restype, argtypes); mirrors include/ppmoe.h
SIGNATURES = {
    "ppmoe_version": (_c_int, []),
    "ppmoe_last_error": (ctypes.c_char_p, []),
    "ppmoe_packed_bytes": (_c_size_t, [_c_int, _c_int, _c_int]),
    "ppmoe_pack": (_c_int, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_int, _c_int, _c_int,
                            _c_void_p, _c_void_p]),
    "ppmoe_workspace_bytes": (_c_size_t, [_c_int, _c_int, _c_int, _c_int]),
    "ppmoe_workspace_init": (_c_int, [_c_void_p, _c_size_t, _c_void_p]),
    "ppmoe_workspace_status": (_c_int, [_c_void_p, _c_void_p]),
    "ppmoe_route_logits": (_c_int, [_c_void_p, _c_int, _c_int, _c_float, _c_void_p, _c_void_p,
                                    _c_void_p]),
    "ppmoe_route_logits_train": (_c_int, [_c_void_p, _c_int, _c_int, _c_float, _c_void_p, _c_void_p,
                                          _c_void_p, _c_void_p]),
    "ppmoe_route_workspace_bytes": (_c_size_t, [_c_int, _c_int, _c_int, _c_int]),
    "ppmoe_route": (_c_int, [_c_void_p, _c_int, _c_void_p, _c_int, _c_int, _c_int, _c_float, _c_void_p,
                             _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_size_t, _c_void_p]),
    "ppmoe_debug_trace": (None, [_c_void_p]),
    "ppmoe_prefill_workspace_bytes": (_c_size_t, [_c_int, _c_int, _c_int, _c_int]),
    "ppmoe_prefill_route": (_c_int, [_c_void_p, _c_int, _c_void_p, _c_int, _c_int, _c_int, _c_float, _c_void_p,
                                     _c_void_p, _c_void_p, _c_void_p, _c_size_t, _c_void_p]),
    "ppmoe_prefill_experts": (_c_int, [_c_void_p, _c_int, _c_void_p, _c_int, _c_int, _c_int, _c_void_p,
                                       _c_void_p, _c_void_p, _c_void_p, _c_size_t, _c_void_p]),
    "ppmoe_ep_combine": (_c_int, [_c_void_p, _c_void_p, _c_int, _c_int, _c_int, _c_void_p, _c_void_p]),
    "ppmoe_ep_combine_bf16": (_c_int, [_c_void_p, _c_void_p, _c_int, _c_int, _c_int, _c_void_p, _c_void_p]),
    "ppmoe_ep_dispatch_workspace_bytes": (_c_size_t, [_c_int, _c_int]),
    "ppmoe_ep_dispatch": (_c_int, [_c_void_p, _c_void_p, _c_int, _c_int, _c_int, _c_int, _c_int, _c_void_p, _c_int,
                                   _c_void_p, _c_void_p, _c_void_p, _c_size_t, _c_void_p]),
    "ppmoe_ep_experts": (_c_int, [_c_void_p, _c_int, _c_int, _c_void_p, _c_int, _c_int, _c_int, _c_int,
                                  _c_void_p, _c_void_p, _c_size_t, _c_void_p]),
    "ppmoe_ep_partial_pitch": (_c_size_t, [_c_int]),
    "ppmoe_ep_combine_f16s": (_c_int, [_c_void_p, _c_int, _c_void_p, _c_int, _c_int, _c_int, _c_void_p, _c_void_p]),
    "ppmoe_prefill": (_c_int, [_c_void_p, _c_int, _c_void_p, _c_int, _c_int, _c_int, _c_float, _c_void_p,
                               _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_size_t, _c_void_p]),
    "ppmoe_decode_noalloc": (_c_int, [_c_void_p, _c_int, _c_void_p, _c_int, _c_int, _c_int, _c_float,
                                      _c_void_p, _c_void_p]),
    "ppmoe_decode_noalloc_status": (_c_int, [_c_void_p]),
    "ppmoe_decode": (_c_int, [_c_void_p, _c_int, _c_void_p, _c_int, _c_int, _c_int, _c_float,
                              _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
                              _c_size_t, _c_int, _c_void_p]),
    "ppmoe_decode_host": (_c_int, [_c_void_p, _c_int, _c_void_p, _c_int, _c_int, _c_int, _c_float,
                                   _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_size_t,
                                   _c_void_p]),
}

_lib = None


class PPMoEError(RuntimeError):
    def __init__(self, fn: str, rc: int, msg: str):
        super().__init__(f"{fn} -> {rc} ({ERR.get(rc, '?')}): {msg}")
        self.rc = rc


def load() -> ctypes.CDLL:
    """Load libppmoe.so once; raises OSError if it is absent (no fallback path exists)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise OSError(f"libppmoe.so not built ({LIB_PATH}); run __graft_entry__.build()")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(lib, name)
            f.restype = res
            f.argtypes = args
        _lib = lib
    return _lib


def call(name: str, *args) -> int:
    """Call an int-returning entry point; raise PPMoEError on a negative status."""
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != 0:
        raise PPMoEError(name, rc, lib.ppmoe_last_error().decode())
    return rc


def ptr(t) -> int | None:
    """Device pointer of a tensor (None for None)."""
    return None if t is None else t.data_ptr()
