"""ctypes binding of ``libocb.so`` (the C ABI declared in ``include/ocb.h``).

There is no CPU fallback: importing the product API without a built library,
or calling it without a CUDA device, raises.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import os

# OCB_LIBRARY selects another build of the same C ABI (e.g. a register-capped
# variant for tuning); the default is the in-tree libocb.so.
LIB_PATH = Path(os.environ.get("OCB_LIBRARY") or (Path(__file__).resolve().parent / "libocb.so"))

c_void_p = ctypes.c_void_p
c_u32 = ctypes.c_uint32
c_u64 = ctypes.c_uint64
c_int = ctypes.c_int
P = ctypes.POINTER

# (name, restype, argtypes) for every symbol of include/ocb.h
SIGNATURES = [
    ("ocb_version", ctypes.c_char_p, []),
    ("ocb_create", c_int, [P(c_void_p), c_int, c_u32]),
    ("ocb_destroy", None, [c_void_p]),
    ("ocb_last_error", ctypes.c_char_p, [c_void_p]),
    ("ocb_set_target", c_int, [c_void_p, ctypes.c_char_p]),
    ("ocb_lex_batch", c_int, [c_void_p, c_void_p, c_void_p, c_u32, P(c_void_p)]),
    ("ocb_tokens_view", c_int, [c_void_p, P(c_u64), P(c_void_p), P(c_void_p),
                                P(c_void_p), P(c_void_p), P(c_void_p)]),
    ("ocb_tokens_free", None, [c_void_p]),
    ("ocb_lex_device", c_int, [c_void_p, c_void_p, c_u64, c_void_p, c_u32,
                               c_void_p, c_void_p, c_void_p, c_u64, c_void_p,
                               c_void_p, c_void_p, c_void_p]),
    ("ocb_preprocess_batch", c_int, [c_void_p, c_void_p, c_void_p, c_u32, P(c_void_p)]),
    ("ocb_text_view", c_int, [c_void_p, P(c_u64), P(c_void_p), P(c_void_p), P(c_void_p),
                              P(c_void_p)]),
    ("ocb_text_free", None, [c_void_p]),
    ("ocb_parse_batch", c_int, [c_void_p, c_void_p, c_void_p, c_u32, P(c_void_p)]),
    ("ocb_optimize_batch", c_int, [c_void_p, c_void_p, c_void_p, c_u32, P(c_void_p)]),
    ("ocb_compile_batch", c_int, [c_void_p, c_void_p, c_void_p, c_u32, P(c_void_p)]),
    ("ocb_verify_batch", c_int, [c_void_p, c_void_p, c_void_p, c_u32, c_int, c_int,
                                 P(c_void_p)]),
    ("ocb_compile_device", c_int, [c_void_p, c_void_p, c_u64, c_void_p, c_u32, c_int,
                                   P(c_void_p), P(c_u64), P(c_void_p), P(c_void_p)]),
    ("ocb_kernel_profile", c_int, [c_void_p, c_int]),
    ("ocb_stream", c_void_p, [c_void_p]),
    ("ocb_kernel_times", c_int, [c_void_p, P(ctypes.c_double), P(c_u64)]),
    ("ocb_lex_device_static", c_int, [c_void_p, c_u64, c_void_p, c_u32, c_void_p,
                                      c_void_p, c_void_p, c_u64, c_void_p, c_void_p,
                                      c_void_p, c_void_p, ctypes.c_char_p, ctypes.c_size_t]),
]

_lib = None


class LibraryMissing(RuntimeError):
    pass


def load() -> ctypes.CDLL:
    """Load ``libocb.so`` (raises LibraryMissing when it was never built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.is_file():
        raise LibraryMissing(
            f"{LIB_PATH} is missing: build it with `python -m opencuda.build`")
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, res, args in SIGNATURES:
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib
