"""Drop-in compile API: ``compile(src) -> ptx`` and ``compile_batch``.

The reference exposes its compile path only as the CLI
``python -m opencuda SRC --emit-ptx`` (``opencuda/__main__.py:13-102``); its
product is the bytes that CLI writes to the ``.ptx`` file.  ``compile`` returns
exactly those bytes (as ``str``) for one source text, and ``compile_batch``
does so for many translation units (TUs) at once, sharded across GPUs.

What runs where:

* ``#include "name"`` resolution is file I/O and stays on the host
  (``resolve_includes``, same policy as ``opencuda/frontend/preprocess.py:125-175``);
  it only runs when include directories are given, as in the reference
  (``preprocess.py:183-184``).
* Everything else -- directives and macros, lexing, parsing, optimization,
  register allocation and PTX text -- runs in ``libocb.so`` on the GPU.  There
  is no CPU fallback: a TU the engine cannot reproduce raises
  ``CompileError`` with status ``unsupported`` rather than being compiled some
  other way.

Errors: where the reference raises (``ParseError``, ``ValueError`` ...),
``compile`` raises ``CompileError`` whose ``exc_type`` names the reference's
exception class; ``compile_batch`` reports it per TU in ``Result``.
"""
from __future__ import annotations

import heapq
import os
import re
import threading
from dataclasses import dataclass
from pathlib import Path
from typing import Iterable, Sequence

import numpy as np

from . import api

DEFAULT_ARCH = "sm_120"          # opencuda/__main__.py:23
INCLUDE_DEPTH_LIMIT = 32         # opencuda/frontend/preprocess.py:122

_STATUS_NAMES = {api.TU_UNSUPPORTED: "unsupported", api.TU_OVERFLOW: "overflow",
                 api.TU_TIMEOUT: "timeout"}


class CompileError(Exception):
    """The TU did not compile.

    ``exc_type`` is the reference's exception class name where the reference
    raises on this input (``"ParseError"``, ``"ValueError"``, ...), else the
    engine's verdict (``"unsupported"``, ``"overflow"``, ``"timeout"``);
    ``status`` is the per-TU status code of ``include/ocb.h``."""

    def __init__(self, exc_type: str, status: int, msg: str = ""):
        super().__init__(f"{exc_type}: {msg}" if msg else exc_type)
        self.exc_type = exc_type
        self.status = status


@dataclass
class Result:
    """One TU of ``compile_batch``: PTX module text, or why there is none."""
    ptx: str | None
    status: int
    exc_type: str | None

    @property
    def ok(self) -> bool:
        return self.status == api.TU_OK


def status_name(status: int) -> str | None:
    if status == api.TU_OK:
        return None
    if 0 < status < 0x100:
        return api.TU_RAISES.get(status, "Exception")
    return _STATUS_NAMES.get(status, f"status {status:#x}")


# ---------------------------------------------------------------------------
# #include "name" resolution (host file I/O)
# ---------------------------------------------------------------------------
_QUOTED = re.compile(r'#\s*include\s+"([^"]+)"')
_ANGLED = re.compile(r'#\s*include\s+<')


def resolve_includes(source: str, include_paths: Sequence[os.PathLike | str],
                     _seen: set[str] | None = None, _depth: int = 0) -> str:
    """Inline quoted includes, the way the reference's preprocessor does
    before it looks at any directive (``preprocess.py:125-175``).

    Per line (split on ``\\n``), after leading whitespace: ``#include "n"``
    is replaced by the text of the first ``dir/n`` that is a file (resolved
    to an absolute path; each absolute path is inlined once per compilation,
    later includes of it become an empty line); an unresolved quoted include
    and every ``#include <...>`` become an empty line.  Included text is
    resolved the same way, 32 levels deep at most: below that a text is kept
    as it is.  Files are read as UTF-8 text with universal newlines, like
    ``Path.read_text``."""
    if _seen is None:
        _seen = set()
    if _depth > INCLUDE_DEPTH_LIMIT:
        return source
    dirs = [Path(d) for d in include_paths]
    lines = source.split("\n")
    for i, line in enumerate(lines):
        head = line.lstrip()
        if not head.startswith("#"):
            continue
        m = _QUOTED.match(head)
        if m is None:
            if _ANGLED.match(head):
                lines[i] = ""
            continue
        hit = next((c for c in ((d / m.group(1)).resolve() for d in dirs) if c.is_file()),
                   None)
        if hit is None or str(hit) in _seen:
            lines[i] = ""
            continue
        _seen.add(str(hit))
        lines[i] = resolve_includes(hit.read_text(encoding="utf-8"), dirs, _seen, _depth + 1)
    return "\n".join(lines)


# ---------------------------------------------------------------------------
# sharding across GPUs
# ---------------------------------------------------------------------------
def partition_lpt(sizes: Sequence[int], n_parts: int) -> list[list[int]]:
    """Byte-balanced greedy LPT: TUs in decreasing size, each to the part with
    the fewest bytes so far (ties: lowest part index).  Each part keeps its
    TUs in decreasing size, so the largest TUs of a GPU start first."""
    n_parts = max(1, int(n_parts))
    order = sorted(range(len(sizes)), key=lambda i: (-int(sizes[i]), i))
    heap = [(0, k) for k in range(n_parts)]      # (bytes so far, part)
    parts: list[list[int]] = [[] for _ in range(n_parts)]
    for i in order:
        load, k = heapq.heappop(heap)
        parts[k].append(i)
        heapq.heappush(heap, (load + int(sizes[i]), k))
    return parts


_ctx_lock = threading.Lock()
_contexts: dict[tuple[int, int], tuple[api.Context, threading.Lock]] = {}


def _context(device: int, slot: int) -> tuple[api.Context, threading.Lock]:
    """The context of (device, slot) with the lock that serialises its use: a
    device listed twice in ``devices`` gets two contexts (two streams), and
    concurrent callers of one context take turns."""
    with _ctx_lock:
        c = _contexts.get((device, slot))
        if c is None:
            c = _contexts[(device, slot)] = (api.Context(device), threading.Lock())
        return c


def _encode(srcs: Iterable[str | bytes]) -> list[bytes]:
    return [s.encode("utf-8", "surrogateescape") if isinstance(s, str) else bytes(s)
            for s in srcs]


def _compile_on(device: int, slot: int, blobs: list[bytes],
                arch: str) -> tuple[bytes, np.ndarray, np.ndarray]:
    ctx, lock = _context(device, slot)
    with lock:
        ctx.set_target(arch)
        tb = ctx.compile_batch(blobs)
    return tb.data, tb.off, tb.status


def compile_batch(srcs: Sequence[str | bytes], *, arch: str = DEFAULT_ARCH,
                  include_paths: Sequence[os.PathLike | str] = (),
                  devices: Sequence[int] | None = None) -> list[Result]:
    """Compile many TUs; ``Result`` i belongs to ``srcs[i]``.

    ``devices``: CUDA device ordinals to shard over (default: device 0).  The
    TUs are split by bytes with greedy LPT, each device compiles its share in
    its own host thread (one context per listed device; the library releases
    the GIL while the GPU works) and the results come back in input order.

    A device whose call fails (a CUDA error, or the library's watchdog giving
    up on a stream that stops making progress) is dropped for the rest of the
    call and its share is split again, by LPT, over the devices that
    succeeded; only when every device has failed does the first error
    propagate."""
    texts = list(srcs)
    if include_paths:
        texts = [resolve_includes(s if isinstance(s, str) else bytes(s).decode("utf-8"),
                                  include_paths) for s in texts]
    blobs = _encode(texts)
    devs = list(devices) if devices else [0]
    out: list[Result | None] = [None] * len(blobs)
    errors: list[BaseException] = []
    live = list(range(len(devs)))          # slots still trusted
    pending = list(range(len(blobs)))      # TUs without a result

    def work(slot: int, idx: list[int], failed: list):
        try:
            if not idx:
                return
            data, off, st = _compile_on(devs[slot], slot, [blobs[i] for i in idx], arch)
            for j, i in enumerate(idx):
                s = int(st[j])
                ptx = (data[int(off[j]):int(off[j + 1])].decode("utf-8", "surrogateescape")
                       if s == api.TU_OK else None)
                out[i] = Result(ptx=ptx, status=s, exc_type=status_name(s))
        except BaseException as ex:  # noqa: BLE001 -- handled on the caller's thread
            failed.append((slot, ex))
            with _ctx_lock:  # a later call starts this slot on a fresh context
                _contexts.pop((devs[slot], slot), None)

    while pending:
        parts = partition_lpt([len(blobs[i]) for i in pending], len(live))
        shares = [(slot, [pending[k] for k in part]) for slot, part in zip(live, parts)]
        failed: list = []
        if len(shares) == 1:
            work(shares[0][0], shares[0][1], failed)
        else:
            threads = [threading.Thread(target=work, args=(slot, idx, failed), daemon=True)
                       for slot, idx in shares]
            for t in threads:
                t.start()
            for t in threads:
                t.join()
        errors.extend(ex for _, ex in failed)
        dead = {slot for slot, _ in failed}
        live = [s for s in live if s not in dead]
        pending = [i for i in pending if out[i] is None]
        if pending and not live:
            raise errors[0]
    return out  # type: ignore[return-value]


def compile(src: str | bytes, *, arch: str = DEFAULT_ARCH,  # noqa: A001 -- the drop-in name
            include_paths: Sequence[os.PathLike | str] = (), device: int = 0) -> str:
    """PTX module text of one source: the bytes ``python -m opencuda X.cu
    --emit-ptx --arch ARCH`` writes (``opencuda/__main__.py:60-85``) when
    ``include_paths`` is what the CLI searches (its ``-I`` list plus the
    source's directory).  Raises ``CompileError`` where the reference raises
    or the engine cannot reproduce it."""
    r = compile_batch([src], arch=arch, include_paths=include_paths, devices=[device])[0]
    if not r.ok:
        raise CompileError(r.exc_type or "error", r.status)
    return r.ptx  # type: ignore[return-value]


def kernel_count(ptx: str) -> int:
    """Kernels in a PTX module text (``.visible .entry`` headers): the count
    the reference CLI prints (``__main__.py:86``)."""
    return sum(1 for ln in ptx.split("\n") if ln.startswith(".visible .entry"))
