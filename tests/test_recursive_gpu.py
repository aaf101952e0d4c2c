"""Recursive __device__ functions on the GPU: compiled to PTX .func bodies
called with call.uni (parser.py:4089-4153, :4392-4435; codegen/emit.py:506-646,
:1744-1776, :3126-3154), including modules of several recursive functions,
whose order in the module follows the reference's set order.  Hand cases and
seeded random call graphs compared with the live reference."""
import pytest

from oracle import ref_runner
from opencuda.api import TU_UNSUPPORTED
from tests._helpers import DEVFUNC_RECURSIVE_CASES, RECURSIVE_CASES, recursive_sources

pytestmark = pytest.mark.gpu

RAISE_STATUS = {"ValueError": 1, "OverflowError": 2, "ParseError": 3, "KeyError": 4}


@pytest.mark.parametrize("stage", ["ir", "opt", "ptx"])
def test_recursive_against_live_reference(ctx, stage):
    srcs = DEVFUNC_RECURSIVE_CASES + RECURSIVE_CASES + recursive_sources(
        400 if stage == "ptx" else 120, 31)
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
