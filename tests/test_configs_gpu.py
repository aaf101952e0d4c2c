"""PTX parity on the benchmark workloads: the register-pressure kernels
(~6,000 statements, ~20k SSA values, peak live ~4k: the allocator's interval
hulls, back-edge extension and FIFO reuse at scale, ``emit.py:115-342``), the
4,096 random kernels and the lognormal-size batch (median 3 KB, sigma 1, the
tail up to ~140 KB TUs).  Every TU is compared byte for byte with the
reference compiler -- live, or through the golden digests of the whole
workload (``python -m oracle.goldens``); TUs where it raises must report the
same exception class, and no TU of these workloads may be ``unsupported``."""
import pytest

from oracle import goldens, ref_runner
from opencuda import synth
from opencuda.api import TU_UNSUPPORTED
from tests._helpers import check_digests

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


def _against_goldens(ctx, name, idx, srcs):
    gold = goldens.load(name)
    if gold is None:
        pytest.skip(f"golden record {name} not made (python -m oracle.goldens {name})")
    tb = ctx.compile_batch(srcs)
    assert not any(int(s) == TU_UNSUPPORTED for s in tb.status)
    texts = [tb.data[int(tb.off[j]):int(tb.off[j + 1])] for j in range(len(srcs))]
    n_ok, n_raise = check_digests(gold, idx, texts, tb.status)
    assert n_ok + n_raise == len(srcs)
    return n_ok, n_raise


def test_register_pressure_all_256(ctx):
    srcs = synth.regpressure_batch(256, seed=4242)
    n_ok, _ = _against_goldens(ctx, "c4", range(256), srcs)
    assert n_ok == 256


def test_random_4096_all(ctx):
    srcs = synth.random_batch(4096, seed=1234)
    _against_goldens(ctx, "c2", range(4096), srcs)


def test_lognormal_every_16th(ctx):
    """16,384 TUs spread over the whole 262,144-kernel batch (every 16th)."""
    idx = list(range(0, 262144, 16))
    srcs = [synth.lognormal_kernel(5678 + i, i) for i in idx]
    _against_goldens(ctx, "c5", idx, srcs)
