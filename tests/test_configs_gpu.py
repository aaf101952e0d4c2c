"""PTX parity on the workload shapes beyond the 4,096-kernel batch: the
register-pressure kernels (~6,000 statements, ~20k SSA values, peak live
~4k: the allocator's interval hulls, back-edge extension and FIFO reuse at
scale, ``emit.py:115-342``) and a sample of the lognormal-size batch (median
3 KB, sigma 1, the tail up to ~100 KB TUs).  Every TU is compared byte for
byte with the live reference compiler; TUs where it raises must report the
same exception class."""
import pytest

from oracle import ref_runner
from opencuda_b200 import synth
from opencuda_b200.api import TU_UNSUPPORTED

pytestmark = pytest.mark.gpu

RAISE_STATUS = {"ValueError": 1, "OverflowError": 2, "ParseError": 3, "KeyError": 4}


def _check(tb, srcs, ref):
    for i, (s, r) in enumerate(zip(srcs, ref)):
        st = int(tb.status[i])
        assert st != TU_UNSUPPORTED, (i, s[:200])
        if "ptx" not in r:
            exc = r.get("raises") or r["error"][0]
            assert st == RAISE_STATUS.get(exc, 6), (i, exc, st)
            continue
        assert st == 0, (i, st, len(s))
        assert tb.text(i) == r["ptx"], (i, len(s))


def test_register_pressure_kernels_full_size(ctx):
    srcs = synth.regpressure_batch(12)
    tb = ctx.compile_batch(srcs)
    with ref_runner.RefPool() as pool:
        ref = pool.run(srcs, what=("ptx",), chunksize=1)
    _check(tb, srcs, ref)


def test_register_pressure_kernels_sizes(ctx):
    srcs = [synth.regpressure_kernel(900 + k, k, n) for k, n in
            enumerate([8, 9, 10, 50, 200, 800, 2000, 3000])]
    tb = ctx.compile_batch(srcs)
    with ref_runner.RefPool() as pool:
        ref = pool.run(srcs, what=("ptx",), chunksize=1)
    _check(tb, srcs, ref)


def test_lognormal_sample(ctx):
    srcs = synth.lognormal_batch(n=1200, seed=5678)
    tb = ctx.compile_batch(srcs)
    with ref_runner.RefPool() as pool:
        ref = pool.run(srcs, what=("ptx",), chunksize=4)
    _check(tb, srcs, ref)
