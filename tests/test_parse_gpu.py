"""GPU parser parity: libocb's sm_100a parser (preprocess -> lex -> parse on
the device) against the reference's parse() -- committed golden IR, and the
live reference (oracle/_ref/py in worker processes on this host) on seeded
generated kernels and token-level mutations of them."""
import pytest

from oracle import ref_runner
from opencuda import synth
from opencuda.api import TU_UNSUPPORTED
from tests._helpers import golden, mutate_sources, PARSE_CASES

pytestmark = pytest.mark.gpu

# exception type -> TU status (include/ocb.h OCB_TU_RAISES_*)
RAISE_STATUS = {"ValueError": 1, "OverflowError": 2, "ParseError": 3, "KeyError": 4,
                "error": 5}


def check_ir(tb, srcs, ref, allow_unsupported=0.0, key="ir"):
    unsup = 0
    for i, (s, r) in enumerate(zip(srcs, ref)):
        st = int(tb.status[i])
        if st == TU_UNSUPPORTED:
            unsup += 1
            continue
        exc = r.get("raises") or (r["error"][0] if "error" in r else None)
        if exc is not None and key not in r:
            assert st == RAISE_STATUS.get(exc, 6), (i, exc, st, s[:300])
            continue
        assert st == 0, (i, st, s[:300])
        assert tb.text(i) == r[key], (i, s[:300])
    assert unsup <= allow_unsupported * len(srcs), unsup


def test_golden_ir(ctx):
    cases = golden("ir_golden.json.gz")["cases"]
    srcs = [c["src"] for c in cases]
    check_ir(ctx.parse_batch(srcs), srcs, cases, allow_unsupported=0.02)


def test_hand_cases_all_supported(ctx):
    tb = ctx.parse_batch(PARSE_CASES)
    assert not any(int(s) == TU_UNSUPPORTED for s in tb.status)


@pytest.mark.parametrize("seed", [3, 4])
def test_generated_kernels_against_live_reference(ctx, seed):
    srcs = [synth.SGEMM_SRC] + synth.random_batch(600, seed=seed)
    tb = ctx.parse_batch(srcs)
    with ref_runner.RefPool() as pool:
        ref = pool.run(srcs, what=("ir",), chunksize=8)
    check_ir(tb, srcs, ref)


def test_mutations_against_live_reference(ctx):
    srcs = mutate_sources(1500, 77)
    tb = ctx.parse_batch(srcs)
    with ref_runner.RefPool() as pool:
        ref = pool.run(srcs, what=("ir",), chunksize=16)
    check_ir(tb, srcs, ref, allow_unsupported=0.02)


# ---- optimizer (optimize.py:1443 optimize, unroll.py) -----------------------

def test_golden_optimized_ir(ctx):
    cases = golden("ir_golden.json.gz")["cases"]
    srcs = [c["src"] for c in cases]
    check_ir(ctx.optimize_batch(srcs), srcs, cases, allow_unsupported=0.02, key="opt")


@pytest.mark.parametrize("seed", [5, 6])
def test_optimized_kernels_against_live_reference(ctx, seed):
    srcs = [synth.SGEMM_SRC] + synth.random_batch(600, seed=seed)
    tb = ctx.optimize_batch(srcs)
    with ref_runner.RefPool() as pool:
        ref = pool.run(srcs, what=("opt",), chunksize=8)
    check_ir(tb, srcs, ref, key="opt")


def test_optimized_mutations_against_live_reference(ctx):
    srcs = mutate_sources(1500, 78)
    tb = ctx.optimize_batch(srcs)
    with ref_runner.RefPool() as pool:
        ref = pool.run(srcs, what=("opt",), chunksize=16)
    check_ir(tb, srcs, ref, allow_unsupported=0.02, key="opt")
