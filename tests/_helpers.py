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
