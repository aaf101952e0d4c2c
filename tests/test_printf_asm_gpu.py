"""printf (lowered to vprintf), inline asm and the texture / surface /
mbarrier intrinsics on the GPU (parser.py:1645-1679, :1732-1738,
:2326-2375; codegen/emit.py:1151-1168, :1661-1740, :1919-1999): hand cases
and seeded kernels compared with the live reference as parsed IR, optimized
IR and PTX."""
import pytest

from oracle import ref_runner
from opencuda.api import TU_UNSUPPORTED
from tests._helpers import PRINTF_ASM_CASES, printf_sources

pytestmark = pytest.mark.gpu

RAISE_STATUS = {"ValueError": 1, "OverflowError": 2, "ParseError": 3, "KeyError": 4}


@pytest.mark.parametrize("stage", ["ir", "opt", "ptx"])
def test_printf_asm_against_live_reference(ctx, stage):
    srcs = PRINTF_ASM_CASES + printf_sources(200, 31)
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
