"""The reference's own kernel corpus (its ``tests/*.cu``) compiled on the GPU.

The fixture ``baseline/_ref/corpus.npz`` is made from the reference checkout
by ``python -m oracle.corpus`` (sources plus the reference's result digests).
Every file must either compile to the reference's bytes, raise the same
exception class, or be reported unsupported; nothing may differ.  The share
of byte-identical files is printed."""
import hashlib
import json

import pytest

from oracle import corpus
from opencuda.api import TU_UNSUPPORTED

pytestmark = pytest.mark.gpu


def test_reference_corpus(ctx):
    fx = corpus.load()
    if fx is None:
        pytest.skip("corpus fixture not made (python -m oracle.corpus)")
    buf, off, names = fx["buf"], fx["off"], fx["names"]
    tb = ctx.compile_batch(buf=buf, tu_off=off)
    c = {"identical": 0, "reference_raises": 0, "unsupported": 0, "mismatched": 0}
    bad, unsup = [], []
    for i in range(len(names)):
        st, gs = int(tb.status[i]), int(fx["status"][i])
        if st == TU_UNSUPPORTED:
            c["unsupported"] += 1
            unsup.append(str(names[i]))
        elif st == 0 and gs == 0 and \
                hashlib.sha256(tb.text(i).encode("utf-8", "surrogateescape")).digest() == \
                bytes(fx["digest"][i]):
            c["identical"] += 1
        elif st != 0 and gs != 0 and st == gs:
            c["reference_raises"] += 1
        else:
            c["mismatched"] += 1
            bad.append((str(names[i]), st, gs))
    c["files"] = len(names)
    c["share_identical_or_same_raise"] = (c["identical"] + c["reference_raises"]) / len(names)
    print("corpus:", json.dumps(c), "unsupported:", " ".join(unsup))
    assert not bad, bad[:10]
