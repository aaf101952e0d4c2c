"""`__device__` functions on the GPU: definitions kept as token ranges and
expanded at each call (parser.py:1749-1929, 4031-4087) -- several returns,
void helpers, nested calls, prototypes and qualifiers, helpers defined after
their callers, `&x` out-parameters spilled to .local, calls the reference's emitter has no
case for -- compared with the live reference as parsed IR, optimized IR
and PTX.  Recursive helpers, which the reference compiles to .func bodies,
are covered by test_recursive_gpu.py."""
import pytest

from oracle import ref_runner
from opencuda.api import TU_UNSUPPORTED
from tests._helpers import (ADDR_OF_CASES, CAST_CASES, DEVFUNC_CASES,
                            ARRAY_PARAM_CASES, HEXFLOAT_CASES, INTRINSIC_CASES,
                            HALF_REDUCE_CASES, MORE_INTRINSIC_CASES, UNKNOWN_CALL_CASES,
                            devfunc_sources)

pytestmark = pytest.mark.gpu

RAISE_STATUS = {"ValueError": 1, "OverflowError": 2, "ParseError": 3, "KeyError": 4}


@pytest.mark.parametrize("stage", ["ir", "opt", "ptx"])
def test_device_functions_against_live_reference(ctx, stage):
    srcs = (DEVFUNC_CASES + ADDR_OF_CASES + UNKNOWN_CALL_CASES + INTRINSIC_CASES + CAST_CASES +
            HEXFLOAT_CASES + ARRAY_PARAM_CASES + MORE_INTRINSIC_CASES + HALF_REDUCE_CASES +
            devfunc_sources(300, 31))
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

