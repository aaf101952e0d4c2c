"""Command line: ``python -m opencuda SRC [SRC ...] --emit-ptx``.

The flags and stdout lines of the reference CLI (``opencuda/__main__.py:13-102``):
``--out``, ``--emit-ptx``, ``--arch`` (default sm_120), ``-I/--include DIR``
(repeatable; the source's own directory is searched last) and ``-v``.  Each
``.ptx`` file holds the bytes the reference writes.  Several sources compile
as one batch on the GPU (``--devices 0,1,...`` shards them across GPUs); a
source that fails is reported on stderr, the others are still written, and
the exit code is 1.

Without ``--emit-ptx`` the reference assembles a cubin with OpenPTXas, a
separate project; that stage is not part of this package, so the CLI says so
and exits 1.
"""
from __future__ import annotations

import argparse
import sys
from pathlib import Path


def _parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(
        prog="opencuda",
        description="B200 batch compiler for OpenCUDA's CUDA-C subset (C to PTX)")
    ap.add_argument("source", nargs="*", help="input .cu file(s)")
    ap.add_argument("--out", default=None, help="output file (one source only)")
    ap.add_argument("--emit-ptx", action="store_true", help="emit PTX text")
    ap.add_argument("--arch", default="sm_120", help="`.target` of the PTX module")
    ap.add_argument("-I", "--include", action="append", default=[], metavar="DIR",
                    help="add a directory to the search path of #include \"...\"")
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--devices", default=None,
                    help="comma-separated CUDA devices to shard the sources over")
    return ap


def main(argv: list[str] | None = None) -> int:
    ap = _parser()
    args = ap.parse_args(argv)
    if not args.source:
        ap.print_help()
        return 0
    if args.out and len(args.source) > 1:
        ap.error("--out takes one source")
    if not args.emit_ptx:
        print("opencuda: cubin output needs OpenPTXas, which is not part of this "
              "package; use --emit-ptx", file=sys.stderr)
        return 1

    from . import compiler

    paths = [Path(s) for s in args.source]
    texts = [p.read_text(encoding="utf-8") for p in paths]
    # The reference searches -I directories first, then the source's own one.
    inc = [Path(d) for d in args.include]
    texts = [compiler.resolve_includes(t, inc + [p.parent]) for t, p in zip(texts, paths)]
    devices = [int(d) for d in args.devices.split(",")] if args.devices else None
    results = compiler.compile_batch(texts, arch=args.arch, devices=devices)

    rc = 0
    for src, p, r in zip(args.source, paths, results):
        print(f"[opencuda] Parsing {src}...")
        if not r.ok:
            print(f"opencuda: {src}: {r.exc_type}", file=sys.stderr)
            rc = 1
            continue
        n = compiler.kernel_count(r.ptx)
        print(f"[opencuda] {n} kernel(s) found")
        out = args.out or str(p.with_suffix(".ptx"))
        Path(out).write_text(r.ptx, encoding="utf-8")
        print(f"[opencuda] Wrote PTX: {out} ({n} kernels)")
        if args.verbose:
            print(r.ptx)
    if rc == 0:
        print("[opencuda] Done.")
    return rc


if __name__ == "__main__":
    sys.exit(main())
