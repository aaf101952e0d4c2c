"""Shared helpers for the test modules."""
from __future__ import annotations

import gzip
import json
import random
from functools import lru_cache
from pathlib import Path

GOLDEN = Path(__file__).resolve().parent / "golden"


@lru_cache(maxsize=None)
def golden(name: str):
    with gzip.open(GOLDEN / name, "rt", encoding="utf-8") as f:
        return json.load(f)


RAISE_CODE = {"ValueError": 1, "OverflowError": 2}


def fuzz_sources(n: int, seed: int, maxlen: int = 80):
    r = random.Random(seed)
    alpha = list("\"'/*\\\n \t\r.0123456789xXeEpP+-fFuUlLabz_=<>&|!;#@\x0c") + [
        "0x1.8p3", "1e+", "'\\n'", "/*", "*/", "//", '"a\\"b"', "0x", "..",
        "1.e5f", "0x.p1", "0x1p1024", "0x1.fffffffffffff8p1023", "int", "for"]
    return ["".join(r.choice(alpha) for _ in range(r.randint(0, maxlen))) for _ in range(n)]


PP_NAMES = ['A', 'B', 'AB', 'F', 'G', 'FG', 'X_1', 'defined', 'N']


def pp_fuzz_sources(n: int, seed: int):
    """Seeded directive-heavy TUs for the preprocessor (no macro whose body
    calls itself: the reference never returns on those)."""
    r = random.Random(seed)
    out = []
    for _ in range(n):
        lines = []
        for _ in range(r.randint(1, 25)):
            k = r.random()
            nm = r.choice(PP_NAMES)
            if k < 0.15:
                lines.append(f"#define {nm} " + r.choice(
                    ['1', 'A + B', '(x)', 'F(1, 2)', 'AB*2', '', 'B', '0x10u', 'A // c', '"s"',
                     'x\\ty', 'q\\n']))
            elif k < 0.25:
                body = r.choice(['a + b', '(a)*2', 'a ## b', '__VA_ARGS__', 'f(a, b)', 'a',
                                 'G(a)', 'x', 'F(a)', 'AB(b)'])
                if body.startswith(nm + '('):
                    body = 'a'
                params = r.choice(['a', 'a, b', 'x, ...', '', ' a , b '])
                lines.append(f"#define {nm}({params}) {body}")
            elif k < 0.30:
                lines.append(f"#undef {nm}")
            elif k < 0.36:
                lines.append(f"#ifdef {nm}")
            elif k < 0.40:
                lines.append(f"#ifndef {nm}")
            elif k < 0.45:
                lines.append("#if " + r.choice(
                    ['1', '0', 'A', 'defined(A)', 'defined B', 'A == 1', 'A && B', '!A',
                     'A + 1 > 2', '1 < 2 < 3', '(A)', '2**3 == 8', '7 // 2 == 3', '1 << 4',
                     'FG', '', '-7 % 3 == 2', '0x1F & 3', '1/0', '3 > 2 > 1']))
            elif k < 0.48:
                lines.append('#elif A')
            elif k < 0.53:
                lines.append(r.choice(['#else', '#endif', '# endif', '#endif // x', '  #  else']))
            elif k < 0.56:
                lines.append(r.choice(['#include "x.h"', '#include <y.h>', '# include "a b"',
                                       '#pragma once', '#line 5', '#error no']))
            elif k < 0.60:
                lines.append(r.choice(['x = A + \\', '  B;', 'y \\', '\\']))
            else:
                lines.append(r.choice(['x = A + B;', 'F(1, 2);', 'FG(A, (B, 3));', 'G(F(1,2))',
                                       'AB = A*B', 's = "A";', 'N(1)', 'F (x)', 'call(F,G)',
                                       'y = AB + FG;', 'defined', 'F("a\\n")', 'G(\'q\')']))
        out.append("\n".join(lines) + r.choice(["", "\n"]))
    return out
