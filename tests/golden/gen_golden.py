"""Regenerates the golden fixtures in this directory from the live reference.

Run here (where the reference checkout exists) after ``oracle/build_ref.sh``:

    python tests/golden/gen_golden.py

The fixtures are small gzip'd JSON files: inputs written by this script (edge
cases, seeded fuzz, seeded synthetic workloads -- no reference test input is
copied) and the reference's outputs for them, produced by the unmodified
reference compiler in ``oracle/_ref/py`` with PYTHONHASHSEED=0.
"""
from __future__ import annotations

import gzip
import json
import random
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

from oracle import ref_runner  # noqa: E402
from opencuda import synth  # noqa: E402

LEX_EDGE = [
    "", "a", "\n", "\n\n\n", "/", "//", "/*", "/**/", "/*/", "/*/*/", "/* */x",
    "/* unterminated\n\n x = 1;", "a/*b*/c", "a//b\nc", "x = 1; // tail",
    '"', '"abc', '"a\\"b"', '"a\\\\"b"', '"\\', '"a\nb"\nc', "s = \"//\" + x;",
    "'", "'a", "'a'", "'\\n'", "'\\''", "''", "'''x'", "'\\'", "'\n'", "'\"'",
    "c = '\"'; d = \"'\";", "'/'/'*'",
    "0x", "0x1", "0x1.", "0x1.8", "0x1.8p3", "0x1.8p3f", "0x1.8P-3L", "0x.8p1",
    "0x.p1", "0xg", "0x1p1024", "0x1.fffffffffffff8p1023",
    "0x1.fffffffffffff7p1023", "0x0p99999", "0x1p-1080",
    "1.", ".5", ".", "..", "...", "1.e5", "1e+", "1e+5f", "1f", "1F", "1.5L",
    "123ull", "7u", "0777", "08", "1..2", "1.5e", "1.5e+", "1.5e+x", "9ex",
    "a.b", "x->y", "a-->b", "<<=", ">>=", "<<", ">>", "<=", ">=", "a<<=b>>=c",
    "++x--", "x+=1-=2*=3/=4%=5&=6|=7^=8", "a&&b||c&d|e^f~g!h", "a==b!=c",
    "(){}[];,.?:", "x\t=\r\n1;", "#define X 1\nX", "a @ b $ c ` d \\ e",
    "\x0c\x0b", "tab\tsep", "__global__ void k() {}", "__forceinline__ _Bool",
    "unsigned long long x = 0xFFFFFFFFFFFFFFFFULL;", "class C; inline register extern",
    "été = 1;", "// é\nx", "/* é */ y",
]


def fuzz(n, seed):
    r = random.Random(seed)
    alpha = list("\"'/*\\\n \t\r.0123456789xXeEpP+-fFuUlLabz_=<>&|!;#@\x0c") + [
        "0x1.8p3", "1e+", "'\\n'", "/*", "*/", "//", '"a\\"b"', "0x", "..",
        "1.e5f", "0x.p1", "0x1p1024", "int", "__global__"]
    return ["".join(r.choice(alpha) for _ in range(r.randint(0, 50))) for _ in range(n)]


def lex_cases():
    cases = list(LEX_EDGE) + fuzz(500, 2024)
    buf, off = synth.lexstress_batch(total_bytes=64 * 1024, tu_bytes=4096, seed=17,
                                     pool_lines=4000)
    cases += [buf[off[i]:off[i + 1]].decode() for i in range(len(off) - 1)]
    cases += [synth.SGEMM_SRC] + synth.random_batch(4, seed=77)
    return cases


PP_EDGE = [
    "", "x", "#define A 1\nA", "#define A 1\n#undef A\nA", "#define F(a,b) a+b\nF(1,2)",
    "#define F(a, b) b a\nF(b, 1)", "#define V(x, ...) f(x, __VA_ARGS__)\nV(1, 2, 3)",
    "#define C(a, b) a ## b\nC(x, y)", "#define S \"A\"\nS A", "#ifdef A\nno\n#else\nyes\n#endif",
    "#if 0\nno\n#elif 1\nelif\n#else\nelse\n#endif", "#if A && B\ntaken\n#endif",
    "#define X 2\n#if X > 1\nbig\n#endif", "#if\nempty\n#endif", "#if(1)\nparen\n#endif",
    "#endif // tail\nx", "a \\\nb", "a \\", "\\", "#define L long \\\n value\nL",
    "#include \"missing.h\"\ny", "#include <stdio.h>\ny", "#  define  SP  7\nSP",
    "#define A B\n#define B A\nA B", "#define A A+1\nA", "#define BAD x\\qy\nBAD",
    "#define NL a\\nb\nNL", "#define F(x) [x]\nF(\"a\\tb\")", "#define F(x) x\nF((1, 2))",
    "#define F(x) x\nF(unbalanced", "#define F (x)\nF", "#define E\n#ifdef E\nE\n#endif",
    "#define AB 1\n#define A 2\nAB A", "#if 1 << -1\nneg\n#endif", "#if 010\noct\n#endif",
    "#define Z // only comment\nZ", "#define F() k\nF() F( )",
]


def pp_cases():
    from tests._helpers import pp_fuzz_sources
    cases = list(PP_EDGE) + pp_fuzz_sources(400, 4242)
    buf, off = synth.lexstress_batch(total_bytes=96 * 1024, tu_bytes=16384, seed=21,
                                     pool_lines=4000)
    cases += [buf[off[i]:off[i + 1]].decode() for i in range(len(off) - 1)]
    cases += [synth.SGEMM_SRC]
    return cases


def ir_cases():
    from tests._helpers import PARSE_CASES, mutate_sources
    return (list(PARSE_CASES) + [synth.SGEMM_SRC] + synth.random_batch(48, seed=99)
            + mutate_sources(300, 4243))


def write(name, obj):
    with gzip.open(HERE / name, "wt", encoding="utf-8") as f:
        json.dump(obj, f)


def main():
    cases = lex_cases()
    with ref_runner.RefPool() as pool:
        toks = pool.lex_raw(cases, chunksize=16)
    out = []
    for src, t in zip(cases, toks):
        if isinstance(t, tuple):
            out.append({"src": src, "raises": t[1]})
        else:
            out.append({"src": src, "tokens": [list(x) for x in t]})
    write("lex_golden.json.gz", {"generator": "tests/golden/gen_golden.py",
                                 "gen_version": synth.GEN_VERSION, "cases": out})
    print(f"lex_golden: {len(out)} cases")
    cases = pp_cases()
    with ref_runner.RefPool() as pool:
        res = pool.run(cases, what=("pp",), chunksize=16)
    out = []
    for src, r in zip(cases, res):
        if "error" in r:
            out.append({"src": src, "raises": r["error"][0]})
        else:
            out.append({"src": src, "pp": r["pp"]})
    write("pp_golden.json.gz", {"generator": "tests/golden/gen_golden.py",
                                "gen_version": synth.GEN_VERSION, "cases": out})
    print(f"pp_golden: {len(out)} cases")
    cases = ir_cases()
    with ref_runner.RefPool() as pool:
        res = pool.run(cases, what=("ir", "opt", "ptx"), chunksize=4)
    out = []
    for src, r in zip(cases, res):
        c = {"src": src}
        for k in ("ir", "opt", "ptx"):
            if k in r:
                c[k] = r[k]
        if "error" in r:
            c["raises"] = r["error"][0]
            c["stage"] = r["error"][2]
        out.append(c)
    write("ir_golden.json.gz", {"generator": "tests/golden/gen_golden.py",
                                "gen_version": synth.GEN_VERSION, "cases": out})
    print(f"ir_golden: {len(out)} cases")


if __name__ == "__main__":
    main()
