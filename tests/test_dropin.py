"""Host side of the drop-in surface, on CPU: include resolution against the
reference's own ``_resolve_includes`` (``preprocess.py:125-175``), the LPT
sharding, the CLI's argument handling, and that the product path fails loudly
when there is no GPU (no CPU fallback)."""
import os
import random
import subprocess
import sys
from pathlib import Path

import pytest

from oracle import ref_runner
from opencuda import compiler

ROOT = Path(__file__).resolve().parent.parent


def _tree(tmp: Path):
    """A small include tree with nesting, a cycle, a shared header, CRLF
    lines, angle-bracket and unresolved includes, and whitespace variants."""
    inc = tmp / "inc"
    sub = tmp / "src"
    inc.mkdir()
    sub.mkdir()
    (inc / "a.h").write_text('#define A 1\n#include "b.h"\nint a_fn;\n')
    (inc / "b.h").write_text('#include "a.h"\n#define B (A+1)\n')         # cycle back to a.h
    (inc / "common.h").write_text("#define COMMON 7\r\nfloat c;\r\n")
    (sub / "local.h").write_text('#include "common.h"\n  #  include   "common.h"\nint local;\n')
    (inc / "deep0.h").write_text("")
    for k in range(40):                                                     # deeper than 32
        (inc / f"deep{k + 1}.h").write_text(f'#include "deep{k}.h"\nint d{k};\n')
    (inc / "ws.h").write_text('\t#include <cuda.h>\n#include"nospace.h"\n#include "missing.h"\n')
    return inc, sub


SOURCES = [
    '#include "a.h"\n__global__ void k(float *x) { x[0] = A + B; }\n',
    '#include "local.h"\n#include "common.h"\n#include <stdio.h>\nint z;',
    '  #include "deep40.h"\n',
    '#include "ws.h"\n#include "a.h"\n#include "a.h"\n',
    "no includes at all\n# include \"b.h\"\n",
    "",
    '#include "sub/../a.h"\n',
]


def test_resolve_includes_matches_reference(tmp_path):
    inc, sub = _tree(tmp_path)
    dirs = [inc, sub]
    with ref_runner.RefPool(2) as pool:
        want = pool.resolve_includes(SOURCES, dirs)
        want_rev = pool.resolve_includes(SOURCES, dirs[::-1])
    for s, w, wr in zip(SOURCES, want, want_rev):
        assert compiler.resolve_includes(s, dirs) == w
        assert compiler.resolve_includes(s, dirs[::-1]) == wr


def test_resolve_includes_random_trees_match_reference(tmp_path):
    r = random.Random(3)
    names = [f"h{k}.h" for k in range(8)]
    d1, d2 = tmp_path / "d1", tmp_path / "d2"
    d1.mkdir()
    d2.mkdir()
    for nm in names:
        for d in (d1, d2):
            if r.random() < 0.6:
                lines = []
                for _ in range(r.randint(0, 6)):
                    k = r.random()
                    if k < 0.4:
                        lines.append(f'{" " * r.randint(0, 2)}#{" " * r.randint(0, 1)}include '
                                     f'"{r.choice(names)}"')
                    elif k < 0.5:
                        lines.append("#include <x.h>")
                    else:
                        lines.append(f"int v{r.randint(0, 99)}; // {d.name}/{nm}")
                (d / nm).write_text("\n".join(lines) + r.choice(["", "\n"]))
    srcs = ["\n".join(f'#include "{r.choice(names)}"' for _ in range(r.randint(0, 5)))
            for _ in range(40)]
    with ref_runner.RefPool(2) as pool:
        want = pool.resolve_includes(srcs, [d1, d2])
    assert [compiler.resolve_includes(s, [d1, d2]) for s in srcs] == want


def test_partition_lpt_balances_and_covers():
    r = random.Random(11)
    sizes = [int(r.lognormvariate(8, 1)) for _ in range(5000)]
    for n in (1, 2, 3, 8):
        parts = compiler.partition_lpt(sizes, n)
        assert sorted(i for p in parts for i in p) == list(range(len(sizes)))
        loads = [sum(sizes[i] for i in p) for p in parts]
        assert max(loads) - min(loads) <= max(sizes)
        for p in parts:
            assert all(sizes[a] >= sizes[b] for a, b in zip(p, p[1:]))
    assert compiler.partition_lpt([], 4) == [[], [], [], []]


def test_status_names():
    assert compiler.status_name(0) is None
    assert compiler.status_name(3) == "ParseError"
    assert compiler.status_name(0x100) == "unsupported"
    assert compiler.status_name(0x200) == "overflow"


def _cli(*args, cwd=None):
    env = dict(os.environ, PYTHONPATH=str(ROOT))
    return subprocess.run([sys.executable, "-m", "opencuda", *map(str, args)],
                          capture_output=True, text=True, cwd=cwd, env=env, timeout=300)


def test_cli_help_and_cubin_path():
    p = _cli()
    assert p.returncode == 0 and "--emit-ptx" in p.stdout
    p = _cli("x.cu")
    assert p.returncode == 1 and "OpenPTXas" in p.stderr


def test_cli_out_takes_one_source():
    p = _cli("a.cu", "b.cu", "--emit-ptx", "--out", "x.ptx")
    assert p.returncode == 2 and "--out takes one source" in p.stderr


def test_product_path_fails_loudly_without_gpu():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from opencuda import OcbError
    with pytest.raises(OcbError):
        compiler.compile("__global__ void k() {}")
