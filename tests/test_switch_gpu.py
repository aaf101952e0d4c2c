"""`switch` (parser.py:3030-3138) on the GPU: hand cases (fallthrough chains,
default anywhere, nested switches, break/continue inside loops, a break
outside any loop) and seeded random switch-heavy kernels, compared with the
live reference at every stage: parsed IR, optimized IR and PTX."""
import pytest

from oracle import ref_runner
from opencuda.api import TU_UNSUPPORTED
from tests._helpers import SWITCH_CASES, switch_sources

pytestmark = pytest.mark.gpu

RAISE_STATUS = {"ValueError": 1, "OverflowError": 2, "ParseError": 3, "KeyError": 4}


@pytest.mark.parametrize("stage", ["ir", "opt", "ptx"])
def test_switch_against_live_reference(ctx, stage):
    srcs = SWITCH_CASES + switch_sources(300, 17)
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
