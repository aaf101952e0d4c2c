"""The reference's own test corpus as a parity fixture.

TEST INFRASTRUCTURE ONLY.  The product never imports this module.

The reference repository keeps ~850 CUDA C kernels under ``tests/*.cu``
(hand-written feature and edge-case probes).  This script reads them from the
reference checkout, compiles each with the live reference exactly as its CLI
does (``opencuda/__main__.py:36-89``, ``oracle/ref_runner.py``), and stores

    names     the file names
    buf, off  the sources, packed back to back (uint8 + uint64 offsets)
    status    0 when the reference writes PTX, else the include/ocb.h code of
              the exception class it raises (6 = other)
    digest    sha256 of the PTX module text (zeros when it raises)

in ``baseline/_ref/corpus.npz``.  That directory is git-ignored (the sources
are the reference's, not this repository's) but travels with the working tree
to the GPU host, where ``tests/test_corpus_gpu.py`` compiles every file with
the engine and reports the byte-identical share.

    python -m oracle.corpus [REFERENCE_DIR] [--procs N]

REFERENCE_DIR defaults to $OCB_REFERENCE_DIR, else /root/reference; without a
checkout there the existing fixture is kept.
"""
from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
OUT = ROOT / "baseline" / "_ref" / "corpus.npz"


def load():
    """The corpus fixture as a dict, or None when it was not made."""
    if not OUT.is_file():
        return None
    z = np.load(OUT)
    return {k: z[k] for k in z.files}


def build(ref_dir: Path, procs: int) -> Path | None:
    from oracle import ref_runner
    files = sorted((ref_dir / "tests").glob("*.cu"))
    if not files:
        print(f"corpus: no reference tests under {ref_dir}; keeping {OUT}", file=sys.stderr)
        return None
    srcs = [f.read_bytes() for f in files]
    texts = [b.decode("utf-8", "surrogateescape") for b in srcs]
    with ref_runner.RefPool(procs) as pool:
        res = pool.digests(texts, what="ptx", chunksize=2)
    off = np.zeros(len(srcs) + 1, np.uint64)
    np.cumsum([len(b) for b in srcs], out=off[1:])
    dg = np.zeros((len(srcs), 32), np.uint8)
    for i, r in enumerate(res):
        if r[1]:
            dg[i] = np.frombuffer(r[1], np.uint8)
    OUT.parent.mkdir(parents=True, exist_ok=True)
    tmp = OUT.with_name(OUT.name + f".{os.getpid()}.tmp.npz")
    np.savez(tmp, names=np.array([f.name for f in files]),
             buf=np.frombuffer(b"".join(srcs), np.uint8), off=off,
             status=np.array([r[0] for r in res], np.int16), digest=dg)
    os.replace(tmp, OUT)
    print(f"corpus: {len(files)} reference kernels -> {OUT}")
    return OUT


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("reference", nargs="?",
                    default=os.environ.get("OCB_REFERENCE_DIR", "/root/reference"))
    ap.add_argument("--procs", type=int, default=len(os.sched_getaffinity(0)))
    args = ap.parse_args(argv)
    build(Path(args.reference), args.procs)


if __name__ == "__main__":
    if str(ROOT) not in sys.path:
        sys.path.insert(0, str(ROOT))
    main()
