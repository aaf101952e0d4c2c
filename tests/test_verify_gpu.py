"""GPU IR verifier parity: ``ocb_verify_batch`` against the reference's
``verify_module`` (``opencuda/ir/verify_ir.py:302``) run live on the same
sources, after parse and after optimize, with and without the reachability
check.  The inputs include break/continue stubs (unreachable blocks), switch
chains, inlined device functions, goto labels and token mutations."""
import pytest

from oracle import ref_runner
from opencuda import synth
from opencuda.api import TU_UNSUPPORTED
from tests._helpers import (PARSE_CASES, devfunc_sources, golden, mutate_sources,
                            switch_sources)

pytestmark = pytest.mark.gpu

RAISE_STATUS = {"ValueError": 1, "OverflowError": 2, "ParseError": 3, "KeyError": 4}


def _sources():
    cases = [c["src"] for c in golden("ir_golden.json.gz")["cases"]]
    return (cases + list(PARSE_CASES) + mutate_sources(400, 5) + switch_sources(200, 3)
            + devfunc_sources(150, 4) + synth.random_batch(50, seed=3))


@pytest.mark.parametrize("optimized,reach", [(False, True), (False, False), (True, True)])
def test_verifier_against_live_reference(ctx, optimized, reach):
    srcs = _sources()
    key = ("verify_opt" if optimized else "verify_ir") + ("_reach" if reach else "")
    tb = ctx.verify_batch(srcs, optimized=optimized, check_reachability=reach)
    with ref_runner.RefPool() as pool:
        ref = pool.run(srcs, what=(key,), chunksize=8)
    n_err = n_unsup = 0
    for i, (s, r) in enumerate(zip(srcs, ref)):
        st = int(tb.status[i])
        if st == TU_UNSUPPORTED:
            n_unsup += 1
            continue
        if key not in r:
            exc = r.get("raises") or r["error"][0]
            assert st == RAISE_STATUS.get(exc, 6), (i, exc, st, s[:200])
            continue
        assert st == 0, (i, st, s[:200])
        assert tb.text(i) == r[key], (i, s[:300])
        n_err += bool(r[key])
    assert n_unsup <= 0.05 * len(srcs)
    if reach and not optimized:
        assert n_err > 50          # the unreachable-stub errors are exercised
