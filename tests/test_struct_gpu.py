"""Structs, unions and the CUDA vector types on the GPU (parser.py:98-128,
:3876-3942 and the StructTy paths of the expression, statement, declaration,
kernel-parameter and inlining code): hand cases and seeded random struct
kernels, compiled to PTX and compared byte for byte with the live reference
(or its exception class)."""
import pytest

from oracle import ref_runner
from opencuda.api import TU_UNSUPPORTED
from tests._helpers import STRUCT_CASES, struct_sources

pytestmark = pytest.mark.gpu

RAISE_STATUS = {"ValueError": 1, "OverflowError": 2, "ParseError": 3, "KeyError": 4}


@pytest.mark.parametrize("stage", ["ir", "opt", "ptx"])
def test_structs_against_live_reference(ctx, stage):
    srcs = STRUCT_CASES + struct_sources(400 if stage == "ptx" else 150, 31)
    fn = {"ir": ctx.parse_batch, "opt": ctx.optimize_batch, "ptx": ctx.compile_batch}[stage]
    tb = fn(srcs)
    with ref_runner.RefPool() as pool:
        ref = pool.run(srcs, what=(stage,), chunksize=4)
    for i, (s, r) in enumerate(zip(srcs, ref)):
        st = int(tb.status[i])
        assert st != TU_UNSUPPORTED, (i, s[:300])
        if stage not in r:
            assert st == RAISE_STATUS.get(r["error"][0], 6), (i, r["error"], st)
            continue
        assert st == 0, (i, st, s[:300])
        assert tb.text(i) == r[stage], (i, s)
