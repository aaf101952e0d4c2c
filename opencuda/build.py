"""Builds the package's CUDA library (``libocb.so``) for sm_100a, in-tree.

``python -m opencuda.build [--force]`` or ``build()``; nvcc
cross-compiles, so no GPU is needed.  Each ``csrc/*.cu`` compiles to its own
object under ``opencuda/_build/`` (in parallel), with nvcc's dependency
files deciding which objects are stale; the objects then link into
``libocb.so``.
"""
from __future__ import annotations

import os
import subprocess
import sys
import time
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB = PKG / "libocb.so"
INCLUDE = PKG.parent / "include"
BUILD = PKG / "_build"

NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-Wno-attributes",
    "--expt-relaxed-constexpr",
]


def sources():
    return sorted(CSRC.glob("*.cu"))


def _deps(dfile: Path) -> list[Path]:
    """Prerequisites listed in a make-style dependency file."""
    try:
        text = dfile.read_text().replace("\\\n", " ")
    except OSError:
        return []
    _, _, rest = text.partition(":")
    return [Path(p) for p in rest.split()]


def _obj_stale(src: Path, obj: Path, dfile: Path) -> bool:
    if not obj.is_file() or not dfile.is_file():
        return True
    t = obj.stat().st_mtime
    for p in [src, *_deps(dfile)]:
        try:
            if p.stat().st_mtime > t:
                return True
        except OSError:
            return True
    return False


def _compile(nvcc: str, src: Path, verbose: bool) -> Path:
    obj = BUILD / (src.stem + ".o")
    dfile = BUILD / (src.stem + ".d")
    tmp = obj.with_suffix(".o.tmp")
    cmd = [nvcc, *NVCC_FLAGS, "-I", str(INCLUDE), "-MD", "-MF", str(dfile),
           "-c", str(src), "-o", str(tmp)]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    t0 = time.time()
    subprocess.run(cmd, check=True)
    os.replace(tmp, obj)
    # the object is as new as the sources it was compiled from: an edit made
    # while nvcc ran leaves it stale
    os.utime(obj, (t0, t0))
    return obj


def build(force: bool = False, verbose: bool = False) -> Path:
    nvcc = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
    BUILD.mkdir(exist_ok=True)
    srcs = sources()
    objs = [BUILD / (s.stem + ".o") for s in srcs]
    stale = [s for s, o in zip(srcs, objs)
             if force or _obj_stale(s, o, BUILD / (s.stem + ".d"))]
    if stale:
        with ThreadPoolExecutor(max_workers=min(len(stale), os.cpu_count() or 4)) as ex:
            list(ex.map(lambda s: _compile(nvcc, s, verbose), stale))
    lib_t = LIB.stat().st_mtime if LIB.is_file() else -1.0
    if stale or any(o.stat().st_mtime > lib_t for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc, "-shared", "-gencode", "arch=compute_100a,code=sm_100a",
               "-Xcompiler", "-fPIC", "-Xlinker", "--no-undefined",
               "-o", str(tmp), *map(str, objs)]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB)
