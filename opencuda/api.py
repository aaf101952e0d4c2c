"""Python host API over the sm_100a batch compiler.

Mirrors the reference's operator API for the compile path
(``opencuda/frontend/lexer.py:258`` ``lex``, ``preprocess.py:178``
``preprocess``, the CLI of ``__main__.py``), in batch form: one call handles
many translation units (TUs) on one GPU.  All work runs in ``libocb.so``;
nothing here computes a result on the CPU except turning token spans into the
reference's ``Token.value`` strings.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import _lib

TOK_HEXFLOAT = 0x80
TOK_EOF = 88

# per-TU status codes (include/ocb.h)
TU_OK = 0
TU_RAISES = {1: "ValueError", 2: "OverflowError", 3: "ParseError", 4: "KeyError",
             5: "re.error", 6: "Exception"}
TU_UNSUPPORTED = 0x100
TU_OVERFLOW = 0x200
TU_TIMEOUT = 0x300


class OcbError(RuntimeError):
    """An API or CUDA error reported by libocb."""


def pack_sources(srcs) -> tuple[np.ndarray, np.ndarray]:
    """list[str|bytes] -> (uint8 buffer, uint64 tu_off[n+1])."""
    bs = [s.encode("utf-8") if isinstance(s, str) else bytes(s) for s in srcs]
    off = np.zeros(len(bs) + 1, dtype=np.uint64)
    if bs:
        np.cumsum(np.fromiter((len(b) for b in bs), dtype=np.uint64, count=len(bs)),
                  out=off[1:])
    buf = np.frombuffer(b"".join(bs), dtype=np.uint8) if bs else np.zeros(0, np.uint8)
    return buf, off


@dataclass
class TokenBatch:
    """Token streams of a batch, struct-of-arrays (host copies)."""
    buf: np.ndarray          # uint8 source bytes the spans point into
    start: np.ndarray        # uint32 byte offset of each token
    kindlen: np.ndarray      # uint32 kind << 24 | len
    line: np.ndarray         # uint32 reference Token.line
    tu_tok_off: np.ndarray   # uint64 [n_tu+1]
    status: np.ndarray       # int32 per-TU status

    @property
    def kind(self) -> np.ndarray:
        return (self.kindlen >> 24).astype(np.uint32)

    @property
    def length(self) -> np.ndarray:
        return self.kindlen & 0xFFFFFF

    def n_tu(self) -> int:
        return len(self.tu_tok_off) - 1

    def tokens(self, i: int):
        """TU i as the reference's (kind, value, line) triples.

        A hex-float token's value is str(float.fromhex(span)) as in
        ``opencuda/frontend/lexer.py:282-284``."""
        lo, hi = int(self.tu_tok_off[i]), int(self.tu_tok_off[i + 1])
        raw = self.buf.tobytes() if not isinstance(self.buf, (bytes, bytearray)) else self.buf
        out = []
        for j in range(lo, hi):
            kl = int(self.kindlen[j])
            k, n, s = kl >> 24, kl & 0xFFFFFF, int(self.start[j])
            v = raw[s:s + n].decode("utf-8", "surrogateescape")
            if k & TOK_HEXFLOAT:
                k &= 0x7F
                v = str(float.fromhex(v.rstrip("fFlL")))
            out.append((k, v, int(self.line[j])))
        return out


@dataclass
class TextBatch:
    """Preprocessed text of a batch (host copies)."""
    data: bytes              # every TU's output back to back
    off: np.ndarray          # uint64 [n_tu+1]
    status: np.ndarray       # int32 per-TU status
    qinclude: np.ndarray     # uint32: a quoted #include line was blanked

    def text(self, i: int) -> str:
        return self.data[int(self.off[i]):int(self.off[i + 1])].decode("utf-8", "surrogateescape")


def _view(p, dt, cnt):
    if cnt == 0 or not p.value:
        return np.zeros(0, dtype=dt)
    nbytes = cnt * np.dtype(dt).itemsize
    c = ctypes.cast(p, ctypes.POINTER(ctypes.c_uint8 * nbytes))
    return np.frombuffer(c.contents, dtype=dt, count=cnt).copy()


class Context:
    """One libocb context on one CUDA device."""

    def __init__(self, device: int = 0):
        self.lib = _lib.load()
        self.device = device
        h = ctypes.c_void_p()
        rc = self.lib.ocb_create(ctypes.byref(h), device, 0)
        if rc != 0:
            raise OcbError(f"ocb_create(device={device}) failed with {rc} "
                           "(no CUDA device, or a driver error)")
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            self.lib.ocb_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001  (interpreter shutdown)
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def _check(self, rc: int, what: str):
        if rc != 0:
            msg = self.lib.ocb_last_error(self.h)
            raise OcbError(f"{what}: {msg.decode() if msg else rc}")

    # ---- lexer -----------------------------------------------------------
    def set_target(self, arch: str) -> None:
        """``.target`` of the PTX modules later compiles write (``--arch``)."""
        if getattr(self, "_target", None) == arch:
            return
        self._check(self.lib.ocb_set_target(self.h, arch.encode("utf-8")), "ocb_set_target")
        self._target = arch

    def lex_batch(self, srcs=None, *, buf=None, tu_off=None) -> TokenBatch:
        """Lex every TU (``lexer.py:258`` ``lex`` per TU)."""
        if srcs is not None:
            buf, tu_off = pack_sources(srcs)
        buf = np.ascontiguousarray(buf, dtype=np.uint8)
        tu_off = np.ascontiguousarray(tu_off, dtype=np.uint64)
        n_tu = len(tu_off) - 1
        out = ctypes.c_void_p()
        src_ptr = buf.ctypes.data if len(buf) else None
        self._check(self.lib.ocb_lex_batch(self.h, src_ptr, tu_off.ctypes.data, n_tu,
                                           ctypes.byref(out)), "ocb_lex_batch")
        try:
            n = ctypes.c_uint64()
            ps = [ctypes.c_void_p() for _ in range(5)]
            self.lib.ocb_tokens_view(out, ctypes.byref(n), *[ctypes.byref(p) for p in ps])
            nt = n.value
            return TokenBatch(buf=buf,
                              start=_view(ps[0], np.uint32, nt),
                              kindlen=_view(ps[1], np.uint32, nt),
                              line=_view(ps[2], np.uint32, nt),
                              tu_tok_off=_view(ps[3], np.uint64, n_tu + 1),
                              status=_view(ps[4], np.int32, n_tu))
        finally:
            self.lib.ocb_tokens_free(out)

    # ---- preprocessor ----------------------------------------------------
    def preprocess_batch(self, srcs=None, *, buf=None, tu_off=None) -> TextBatch:
        """Preprocess every TU (``preprocess.py:178`` as the CLI calls it)."""
        return self._text_call("ocb_preprocess_batch", srcs, buf, tu_off)

    def parse_batch(self, srcs=None, *, buf=None, tu_off=None) -> TextBatch:
        """Preprocess, lex and parse every TU (``parser.py:4446 parse``); each
        TU's text is its IR in the canonical line format."""
        return self._text_call("ocb_parse_batch", srcs, buf, tu_off)

    def optimize_batch(self, srcs=None, *, buf=None, tu_off=None) -> TextBatch:
        """As parse_batch, then ``optimize.py:1443 optimize``; each TU's text is
        its optimized IR."""
        return self._text_call("ocb_optimize_batch", srcs, buf, tu_off)

    def compile_batch(self, srcs=None, *, buf=None, tu_off=None) -> TextBatch:
        """Compile every TU to its PTX module text (the reference CLI's
        ``--emit-ptx`` output, ``__main__.py:36-85``)."""
        return self._text_call("ocb_compile_batch", srcs, buf, tu_off)

    def verify_batch(self, srcs=None, *, buf=None, tu_off=None, optimized: bool = False,
                     check_reachability: bool = True) -> TextBatch:
        """Preprocess, lex, parse (and optionally optimize) every TU and check
        its IR with the reference's verifier (``opencuda/ir/verify_ir.py:302``
        ``verify_module``); each TU's text lists the violations per kernel
        (empty when the IR is clean)."""
        return self._text_call("ocb_verify_batch", srcs, buf, tu_off,
                               1 if optimized else 0, 1 if check_reachability else 0)

    def _text_call(self, fn, srcs, buf, tu_off, *extra) -> TextBatch:
        if srcs is not None:
            buf, tu_off = pack_sources(srcs)
        buf = np.ascontiguousarray(buf, dtype=np.uint8)
        tu_off = np.ascontiguousarray(tu_off, dtype=np.uint64)
        n_tu = len(tu_off) - 1
        out = ctypes.c_void_p()
        src_ptr = buf.ctypes.data if len(buf) else None
        self._check(getattr(self.lib, fn)(self.h, src_ptr, tu_off.ctypes.data, n_tu, *extra,
                                          ctypes.byref(out)), fn)
        try:
            n = ctypes.c_uint64()
            ps = [ctypes.c_void_p() for _ in range(4)]
            self.lib.ocb_text_view(out, ctypes.byref(n), *[ctypes.byref(p) for p in ps])
            data = ctypes.string_at(ps[0], n.value) if n.value else b""
            return TextBatch(data=data, off=_view(ps[1], np.uint64, n_tu + 1),
                             status=_view(ps[2], np.int32, n_tu),
                             qinclude=_view(ps[3], np.uint32, n_tu))
        finally:
            self.lib.ocb_text_free(out)

    def compile_device(self, d_src: int, n_bytes: int, d_tu_off: int, n_tu: int,
                       stage: int = 2):
        """Device-pointer form of parse/optimize/compile_batch
        (``ocb_compile_device``, stage 0/1/2).  Returns
        ``(d_out, out_bytes, d_out_off, d_status)``: device addresses owned by
        the context, valid until its next call; the work is complete."""
        d_out, d_off, d_st = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_void_p()
        nb = ctypes.c_uint64()
        self._check(self.lib.ocb_compile_device(self.h, d_src, n_bytes, d_tu_off, n_tu, stage,
                                                ctypes.byref(d_out), ctypes.byref(nb),
                                                ctypes.byref(d_off), ctypes.byref(d_st)),
                    "ocb_compile_device")
        return d_out.value or 0, nb.value, d_off.value or 0, d_st.value or 0

    KERNELS = ("k_cc_parse", "k_cc_opt", "k_cc_emit")

    @property
    def stream(self) -> int:
        """The context's CUDA stream handle (every batch call queues work on it)."""
        return self.lib.ocb_stream(self.h) or 0

    def kernel_profile(self, enable: bool = True) -> None:
        """Zero the per-kernel event timers and switch them on/off."""
        self._check(self.lib.ocb_kernel_profile(self.h, 1 if enable else 0),
                    "ocb_kernel_profile")

    def kernel_times(self) -> dict:
        """``{kernel: (total_ms, launches)}`` since ``kernel_profile(True)``."""
        ms = (ctypes.c_double * 3)()
        n = (ctypes.c_uint64 * 3)()
        self.lib.ocb_kernel_times(self.h, ms, n)
        return {k: (ms[i], n[i]) for i, k in enumerate(self.KERNELS)}

    def lex_device(self, d_src: int, n_bytes: int, d_tu_off: int, n_tu: int,
                   d_start: int, d_kindlen: int, d_line: int, tok_cap: int,
                   d_tu_tok_off: int, d_status: int, d_n_tok: int, stream: int = 0):
        """Device-pointer form (``ocb_lex_device``); queues work on `stream`."""
        self._check(self.lib.ocb_lex_device(self.h, d_src, n_bytes, d_tu_off, n_tu,
                                            d_start, d_kindlen, d_line, tok_cap,
                                            d_tu_tok_off, d_status, d_n_tok, stream),
                    "ocb_lex_device")


_default: dict[int, Context] = {}


def context(device: int = 0) -> Context:
    if device not in _default:
        _default[device] = Context(device)
    return _default[device]


def lex_batch(srcs, device: int = 0) -> TokenBatch:
    return context(device).lex_batch(srcs)


def preprocess_batch(srcs, device: int = 0) -> TextBatch:
    return context(device).preprocess_batch(srcs)


def parse_batch(srcs, device: int = 0) -> TextBatch:
    return context(device).parse_batch(srcs)


def optimize_batch(srcs, device: int = 0) -> TextBatch:
    return context(device).optimize_batch(srcs)


def compile_batch(srcs, device: int = 0) -> TextBatch:
    return context(device).compile_batch(srcs)
