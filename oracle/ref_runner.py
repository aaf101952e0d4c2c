"""Live reference oracle: runs the unmodified reference compiler.

TEST INFRASTRUCTURE ONLY.  Nothing in the product imports this module; only
``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline / reference legs of
``bench.py`` use it, as the checker and as the timed CPU baseline.

The reference (garrick247/opencuda, pure Python) is installed into
``oracle/_ref/py`` by ``oracle/build_ref.sh``.  Its top-level package is also
called ``opencuda``, which clashes with this repository's drop-in package, so
it only ever runs inside ``spawn``-started worker processes whose ``sys.path``
starts with ``oracle/_ref/py`` and does not contain the repository root.
Workers run with ``PYTHONHASHSEED=0`` because the reference's output for TUs
with several recursive ``__device__`` functions depends on set iteration order
(``opencuda/frontend/parser.py:4396-4435``).

Each compile job mirrors the CLI ``python -m opencuda X.cu --emit-ptx``
(``opencuda/__main__.py:36-89``): preprocess with an include path list that
holds one empty directory (the CLI always passes the source's own directory,
``__main__.py:39-44``), parse, optimize, ``ir_to_ptx``, then the module-text
assembly of ``__main__.py:60-85``.
"""
from __future__ import annotations

import os
import sys
import time
import tempfile
import multiprocessing as mp
from pathlib import Path

HERE = Path(__file__).resolve().parent
REF_DIR = HERE / "_ref" / "py"
REPO_ROOT = HERE.parent

_EMPTY_INC = None


def available() -> bool:
    return (REF_DIR / "opencuda" / "frontend" / "lexer.py").is_file()


def _worker_init():
    global _EMPTY_INC
    root = str(REPO_ROOT)
    sys.path[:] = [p for p in sys.path
                   if p not in ("", ".") and os.path.abspath(p) != root]
    sys.path.insert(0, str(REF_DIR))
    for m in list(sys.modules):
        if m == "opencuda" or m.startswith("opencuda."):
            del sys.modules[m]
    import opencuda.frontend.preprocess  # noqa: F401  (warm import)
    import opencuda.frontend.parser  # noqa: F401
    import opencuda.ir.optimize  # noqa: F401
    import opencuda.codegen.emit  # noqa: F401
    import importlib.util
    spec = importlib.util.spec_from_file_location("oracle_ir_dump", HERE / "ir_dump.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    sys.modules["oracle_ir_dump"] = mod
    _EMPTY_INC = tempfile.mkdtemp(prefix="ocb-empty-inc-")


def assemble(ptx_map: dict, arch: str) -> str:
    """Module text exactly as ``__main__.py:60-85`` writes it."""
    out = [".version 9.0", f".target {arch}", ".address_size 64", ""]
    if "__preamble__" in ptx_map:
        out.extend(ptx_map["__preamble__"].split("\n"))
        out.append("")
    for name, text in ptx_map.items():
        if name.startswith("__"):
            continue
        lines = text.split("\n")
        start = 0
        for j, line in enumerate(lines):
            if line.startswith(".visible") or line.startswith("{"):
                start = j
                break
        out.extend(lines[start:])
        out.append("")
    return "\n".join(out)


def _job(args):
    """One TU through the reference.  ``what`` selects the outputs."""
    src, what, arch = args
    from opencuda.frontend.preprocess import preprocess
    from opencuda.frontend.lexer import lex
    res = {}
    try:
        pp = preprocess(src, include_paths=[Path(_EMPTY_INC)])
    except Exception as e:  # noqa: BLE001  (the reference raises arbitrary types)
        res["error"] = [type(e).__name__, str(e)[:200], "preprocess"]
        return res
    if "pp" in what:
        res["pp"] = pp
    if "tok" in what:
        try:
            res["tok"] = [(t.kind.value, t.value, t.line) for t in lex(pp)]
        except Exception as e:  # noqa: BLE001
            res["error"] = [type(e).__name__, str(e)[:200], "lex"]
            return res
    if "ir" in what or "opt" in what:
        from opencuda.frontend.parser import parse
        from opencuda.ir.optimize import optimize
        from oracle_ir_dump import dump_module
        try:
            module = parse(pp)
            if "ir" in what:
                res["ir"] = dump_module(module)
            if "opt" in what:
                res["opt"] = dump_module(optimize(module))
        except Exception as e:  # noqa: BLE001
            res["error"] = [type(e).__name__, str(e)[:200], "parse"]
            return res
    vkeys = [w for w in what if w.startswith("verify")]
    if vkeys:
        # verify_ir / verify_opt (+ "_reach": check_reachability=True)
        from opencuda.frontend.parser import parse
        from opencuda.ir.optimize import optimize
        from oracle_ir_dump import verify_text
        try:
            for w in vkeys:
                module = parse(pp)
                if w.startswith("verify_opt"):
                    module = optimize(module)
                res[w] = verify_text(module, w.endswith("_reach"))
        except Exception as e:  # noqa: BLE001
            res["error"] = [type(e).__name__, str(e)[:200], "verify"]
            return res
    if "ptx" in what:
        from opencuda.frontend.parser import parse
        from opencuda.ir.optimize import optimize
        from opencuda.codegen.emit import ir_to_ptx
        try:
            module = parse(pp)
            module = optimize(module)
            res["ptx"] = assemble(ir_to_ptx(module), arch)
        except Exception as e:  # noqa: BLE001
            res["error"] = [type(e).__name__, str(e)[:200], "compile"]
    return res


def _lex_raw(src):
    """The reference lexer on unpreprocessed text: (kind, value, line)."""
    from opencuda.frontend.lexer import lex
    try:
        return [(t.kind.value, t.value, t.line) for t in lex(src)]
    except Exception as e:  # noqa: BLE001
        return ("error", type(e).__name__, str(e)[:200])


def _lex_only(src):
    from opencuda.frontend.lexer import lex
    try:
        return len(lex(src))
    except Exception:  # noqa: BLE001
        return 0


# exception class of the reference -> per-TU status code of include/ocb.h
RAISE_STATUS = {"ValueError": 1, "OverflowError": 2, "ParseError": 3, "KeyError": 4,
                "error": 5}


def _digest_job(args):
    """One TU through the reference CLI path, reduced to what a parity check
    of many TUs needs: (status code, sha256 of the PTX module text, its byte
    length).  The status is 0 when the reference writes PTX, else the
    ``include/ocb.h`` code of the exception class it raises (6 for others)."""
    import hashlib
    src, what, arch = args
    r = _job((src, what, arch))
    key = "ptx" if "ptx" in what else "pp"
    if key in r:
        b = r[key].encode("utf-8", "surrogateescape")
        return 0, hashlib.sha256(b).digest(), len(b)
    return RAISE_STATUS.get(r["error"][0], 6), b"", 0


def _compile_only(src):
    r = _job((src, ("ptx",), "sm_120"))
    return len(r.get("ptx", ""))


def _resolve(args):
    """The reference's include resolution (``preprocess.py:125-175``)."""
    src, dirs = args
    from opencuda.frontend.preprocess import _resolve_includes
    try:
        return _resolve_includes(src, [Path(d) for d in dirs], visited=set())
    except Exception as e:  # noqa: BLE001
        return ("error", type(e).__name__)


def run_cli(argv, cwd=None, timeout=600):
    """The reference CLI ``python -m opencuda ARGV`` in a fresh interpreter
    (``PYTHONHASHSEED=0``, only ``oracle/_ref/py`` on the path).  Returns
    ``(returncode, stdout, stderr)``."""
    import subprocess
    if not available():
        raise RuntimeError("reference oracle not built: run oracle/build_ref.sh")
    env = dict(os.environ, PYTHONHASHSEED="0", PYTHONPATH=str(REF_DIR))
    p = subprocess.run([sys.executable, "-m", "opencuda", *map(str, argv)], cwd=cwd, env=env,
                       capture_output=True, text=True, timeout=timeout)
    return p.returncode, p.stdout, p.stderr


class RefPool:
    """A pool of spawn workers that run the reference."""

    def __init__(self, processes: int | None = None):
        if not available():
            raise RuntimeError(
                "reference oracle not built: run oracle/build_ref.sh")
        os.environ["PYTHONHASHSEED"] = "0"
        self.processes = processes or len(os.sched_getaffinity(0))
        ctx = mp.get_context("spawn")
        self.pool = ctx.Pool(self.processes, initializer=_worker_init)

    def run(self, srcs, what=("ptx",), arch="sm_120", chunksize=4):
        return self.pool.map(_job, [(s, tuple(what), arch) for s in srcs],
                             chunksize=chunksize)

    def digests(self, srcs, what="ptx", arch="sm_120", chunksize=16):
        """``_digest_job`` over ``srcs`` (``what``: "ptx" or "pp")."""
        return self.pool.map(_digest_job, [(s, (what,), arch) for s in srcs],
                             chunksize=chunksize)

    def resolve_includes(self, srcs, dirs):
        return self.pool.map(_resolve, [(s, [str(d) for d in dirs]) for s in srcs])

    def lex_raw(self, srcs, chunksize=16):
        return self.pool.map(_lex_raw, srcs, chunksize=chunksize)

    def time_compile(self, srcs, chunksize=4):
        """Wall seconds for the reference to compile ``srcs`` to PTX text."""
        t0 = time.perf_counter()
        n = self.pool.map(_compile_only, srcs, chunksize=chunksize)
        return time.perf_counter() - t0, sum(n)

    def time_lex(self, srcs, chunksize=1):
        """Wall seconds for the reference's lex() over ``srcs``."""
        t0 = time.perf_counter()
        n = self.pool.map(_lex_only, srcs, chunksize=chunksize)
        return time.perf_counter() - t0, sum(n)

    def close(self):
        self.pool.terminate()
        self.pool.join()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def tokkind_table() -> dict:
    """Name -> value of the reference's ``TokKind`` (``lexer.py:11-109``)."""
    with RefPool(1) as p:
        return p.pool.apply(_tokkinds)


def _tokkinds():
    from opencuda.frontend.lexer import TokKind
    return {k.name: k.value for k in TokKind}
