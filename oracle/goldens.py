"""Golden digests of the reference compiler's output on the benchmark workloads.

TEST INFRASTRUCTURE ONLY.  The product never imports this module; ``bench.py``
and the GPU tests read the files it writes, as the parity checker.

The seeded workloads of ``opencuda.synth`` are far too large to keep the
reference's output text (the 262,144-kernel lognormal batch alone compiles to
several GB of PTX), and compiling them with the reference takes an hour of CPU
time.  So each TU's reference result is reduced, once, to a digest record:

    status    int16   0 = the reference writes PTX; else the include/ocb.h
                      code of the exception class it raises (6 = other)
    digest    u8[32]  sha256 of the PTX module text (the bytes the CLI
                      ``python -m opencuda X.cu --emit-ptx`` writes,
                      ``opencuda/__main__.py:60-85``) or, for ``c3pp``, of
                      the preprocessed text (``preprocess.py:178``)
    nbytes    int64   length of that text
    src       u8[8]   first 8 bytes of sha256 of the TU source, so that a
                      reader can tell that its generator made the same TU

stored as ``baseline/_ref/goldens/<workload>_g<GEN_VERSION>.npz`` (git-ignored;
it travels with the working tree to the GPU host).  The reference runs from
``oracle/_ref/py`` in spawn workers with ``PYTHONHASHSEED=0``
(``oracle/ref_runner.py``).  Work is saved in parts, so an interrupted run
resumes where it stopped.

    python -m oracle.goldens c5 c2 c4 c3pp [--procs N]
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
OUT = ROOT / "baseline" / "_ref" / "goldens"
PART = 8192


def _workloads():
    from opencuda import synth
    return {
        # 262,144 lognormal-size kernels (median 3 KB, sigma 1)
        "c5": dict(what="ptx", n=262144,
                   make=lambda procs: synth.lognormal_batch(262144, seed=5678, procs=procs)),
        # 4,096 random kernels of 50-200 statements
        "c2": dict(what="ptx", n=4096, make=lambda procs: synth.random_batch(4096, seed=1234)),
        # 256 register-pressure kernels (~20k SSA values each)
        "c4": dict(what="ptx", n=256, make=lambda procs: synth.regpressure_batch(256, seed=4242)),
        # 1 GiB of preprocessor/lexer stress text in 16 KiB TUs
        "c3pp": dict(what="pp", n=None, make=lambda procs: _lexstress_tus()),
    }


def _lexstress_tus():
    from opencuda import synth
    buf, off = synth.lexstress_batch(total_bytes=1 << 30, tu_bytes=16384, seed=99)
    return [buf[int(off[i]):int(off[i + 1])].decode("ascii") for i in range(len(off) - 1)]


def path(name: str) -> Path:
    from opencuda import synth
    return OUT / f"{name}_g{synth.GEN_VERSION}.npz"


def src_digests(srcs) -> np.ndarray:
    out = np.zeros((len(srcs), 8), np.uint8)
    for i, s in enumerate(srcs):
        b = s.encode("utf-8") if isinstance(s, str) else bytes(s)
        out[i] = np.frombuffer(hashlib.sha256(b).digest()[:8], np.uint8)
    return out


def load(name: str):
    """The golden record of workload ``name``, or None when it was not made."""
    p = path(name)
    if not p.is_file():
        return None
    z = np.load(p)
    return {k: z[k] for k in z.files}


def build(name: str, procs: int) -> Path:
    from oracle import ref_runner
    from opencuda import synth
    spec = _workloads()[name]
    t0 = time.time()
    srcs = spec["make"](procs)
    n = len(srcs)
    parts_dir = OUT / f"{name}_g{synth.GEN_VERSION}.parts"
    parts_dir.mkdir(parents=True, exist_ok=True)
    print(f"goldens {name}: {n} TUs, {sum(len(s) for s in srcs)} bytes, generated in "
          f"{time.time() - t0:.0f} s", flush=True)
    with ref_runner.RefPool(procs) as pool:
        for lo in range(0, n, PART):
            hi = min(n, lo + PART)
            pf = parts_dir / f"{lo:08d}.npz"
            if pf.is_file():
                continue
            t1 = time.time()
            res = pool.digests(srcs[lo:hi], what=spec["what"], chunksize=4)
            st = np.array([r[0] for r in res], np.int16)
            dg = np.zeros((hi - lo, 32), np.uint8)
            for j, r in enumerate(res):
                if r[1]:
                    dg[j] = np.frombuffer(r[1], np.uint8)
            nb = np.array([r[2] for r in res], np.int64)
            np.savez(pf, status=st, digest=dg, nbytes=nb)
            print(f"  [{lo}, {hi}) in {time.time() - t1:.0f} s", flush=True)
    st, dg, nb = [], [], []
    for lo in range(0, n, PART):
        z = np.load(parts_dir / f"{lo:08d}.npz")
        st.append(z["status"])
        dg.append(z["digest"])
        nb.append(z["nbytes"])
    meta = {"workload": name, "what": spec["what"], "n": n,
            "gen_version": synth.GEN_VERSION, "made": time.strftime("%Y-%m-%dT%H:%M:%SZ",
                                                                      time.gmtime())}
    out = path(name)
    np.savez(out, status=np.concatenate(st), digest=np.concatenate(dg),
             nbytes=np.concatenate(nb), src=src_digests(srcs),
             meta=np.array(json.dumps(meta)))
    for f in parts_dir.iterdir():
        f.unlink()
    parts_dir.rmdir()
    print(f"goldens {name}: wrote {out} in {time.time() - t0:.0f} s", flush=True)
    return out


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("names", nargs="+", choices=sorted(_workloads()))
    ap.add_argument("--procs", type=int, default=len(os.sched_getaffinity(0)))
    args = ap.parse_args(argv)
    for nm in args.names:
        if path(nm).is_file():
            print(f"goldens {nm}: {path(nm)} exists")
            continue
        build(nm, args.procs)


if __name__ == "__main__":
    if str(ROOT) not in sys.path:
        sys.path.insert(0, str(ROOT))
    main()
