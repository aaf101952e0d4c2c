"""Module-level `__device__` and `__constant__` variables on the GPU
(parser.py:4155-4191, 4305-4366; emit.py:1169-1178, 3164-3190): scalar and
array symbols in both qualifier orders, initializers skipped as the
reference skips them, reads through the symbol, writes and compound
assignments through its address, `&sym` / `&sym[i]` for atomics, symbols
declared after the kernel that reads them, and the `.visible .global/.const`
declarations that lead the module text.  Compared with the live reference as
parsed IR, optimized IR and PTX, and through the drop-in `compile()` call."""
import pytest

import opencuda as oc
from oracle import ref_runner
from tests._helpers import GLOBAL_2D_CASES, GLOBAL_VAR_CASES

pytestmark = pytest.mark.gpu

RAISE_STATUS = {"ValueError": 1, "OverflowError": 2, "ParseError": 3, "KeyError": 4}


@pytest.mark.parametrize("stage", ["ir", "opt", "ptx"])
def test_module_variables_against_live_reference(ctx, stage):
    srcs = GLOBAL_VAR_CASES
    fn = {"ir": ctx.parse_batch, "opt": ctx.optimize_batch, "ptx": ctx.compile_batch}[stage]
    tb = fn(srcs)
    with ref_runner.RefPool() as pool:
        ref = pool.run(srcs, what=(stage,))
    for i, r in enumerate(ref):
        assert stage in r, (i, r.get("error"))
        assert int(tb.status[i]) == 0, (i, int(tb.status[i]))
        assert tb.text(i) == r[stage], (i, srcs[i])


def test_module_variable_declarations_through_compile():
    with ref_runner.RefPool() as pool:
        ref = pool.run(GLOBAL_VAR_CASES, what=("ptx",))
    for src, r in zip(GLOBAL_VAR_CASES, ref):
        ptx = oc.compile(src)
        assert ptx == r["ptx"]
        assert ptx.split("\n")[4].startswith(".visible .")


@pytest.mark.parametrize("stage", ["ir", "opt", "ptx"])
def test_multi_dimensional_module_arrays_against_live_reference(ctx, stage):
    """`__device__ T g[R][C]` carries a row stride that only the element
    lvalue `g[i][j] = v` uses (the rvalue path looks the stride up under the
    address value's name, as the reference does); a `__constant__` array reads
    one dimension and the module loop skips the rest.  Where the reference
    raises, the engine must report the same exception class."""
    srcs = GLOBAL_2D_CASES
    fn = {"ir": ctx.parse_batch, "opt": ctx.optimize_batch, "ptx": ctx.compile_batch}[stage]
    tb = fn(srcs)
    with ref_runner.RefPool() as pool:
        ref = pool.run(srcs, what=(stage,))
    for i, r in enumerate(ref):
        st = int(tb.status[i])
        if stage not in r:
            assert st == RAISE_STATUS.get(r["error"][0], 6), (i, r["error"], st)
            continue
        assert st == 0, (i, st)
        assert tb.text(i) == r[stage], (i, srcs[i])
