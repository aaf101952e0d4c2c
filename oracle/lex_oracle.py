"""ctypes wrapper of the C lexer restatement (``oracle/lex_oracle.c``).

TEST INFRASTRUCTURE ONLY: used by ``tests/`` as the checker of the GPU lexer
and by ``bench.py``'s CPU-baseline leg.  Build with ``make -C oracle``.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

_LIB = Path(__file__).resolve().parent / "_ref" / "liblexoracle.so"
_lib = None

# TokKind values of the reference (opencuda/frontend/lexer.py:11-109).
K_FLOAT = 2
K_EOF = 88
HEXFLOAT_FLAG = 0x80


def _load():
    global _lib
    if _lib is None:
        if not _LIB.is_file():
            raise RuntimeError(f"lexer oracle not built ({_LIB}): make -C oracle")
        lib = ctypes.CDLL(str(_LIB))
        lib.oracle_lex_batch.restype = ctypes.c_int64
        lib.oracle_lex_batch.argtypes = [
            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint32,
            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
            ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p]
        _lib = lib
    return _lib


def lex_batch(buf, tu_off):
    """Lex every TU.

    Returns (start u32, kindlen u32, line u32, tu_tok_off u64, status i32):
    status[i] = 1 / 2 where the reference's lex() raises ValueError /
    OverflowError on a hex float of TU i, else 0."""
    lib = _load()
    tu_off = np.ascontiguousarray(tu_off, dtype=np.uint64)
    src = np.frombuffer(buf, dtype=np.uint8) if isinstance(buf, (bytes, bytearray)) \
        else np.ascontiguousarray(buf, dtype=np.uint8)
    if len(src) == 0:
        src = np.zeros(1, np.uint8)
    n_tu = len(tu_off) - 1
    cap = int(tu_off[-1]) + n_tu + 16
    start = np.empty(cap, dtype=np.uint32)
    kl = np.empty(cap, dtype=np.uint32)
    line = np.empty(cap, dtype=np.uint32)
    tto = np.empty(n_tu + 1, dtype=np.uint64)
    status = np.empty(max(n_tu, 1), dtype=np.int32)
    n = lib.oracle_lex_batch(src.ctypes.data, tu_off.ctypes.data, n_tu,
                             start.ctypes.data, kl.ctypes.data, line.ctypes.data,
                             tto.ctypes.data, cap, status.ctypes.data)
    if n < 0:
        raise RuntimeError("oracle lexer: capacity exceeded")
    return start[:n], kl[:n], line[:n], tto, status[:n_tu]


def as_reference_tokens(buf, start, kindlen, line, lo, hi):
    """Tokens [lo, hi) as the reference's (kind, value, line) triples.

    A hex-float token's value is ``str(float.fromhex(span))`` exactly as the
    reference computes it (``opencuda/frontend/lexer.py:282-284``)."""
    raw = bytes(buf) if not isinstance(buf, (bytes, bytearray)) else buf
    out = []
    for i in range(lo, hi):
        k = int(kindlen[i]) >> 24
        ln = int(kindlen[i]) & 0xFFFFFF
        s = int(start[i])
        val = raw[s:s + ln].decode("utf-8", "surrogateescape")
        if k & HEXFLOAT_FLAG:
            k &= 0x7F
            val = str(float.fromhex(val.rstrip("fFlL")))
        out.append((k, val, int(line[i])))
    return out
