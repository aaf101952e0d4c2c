"""The C lexer restatement (oracle/lex_oracle.c) against the reference's own
token streams (tests/golden/lex_golden.json.gz, generated from the live
reference by tests/golden/gen_golden.py).  CPU only."""
import numpy as np
import pytest

from oracle import lex_oracle
from opencuda import synth
from tests._helpers import golden, RAISE_CODE


@pytest.fixture(scope="module")
def oracle_run():
    cases = golden("lex_golden.json.gz")["cases"]
    buf, off = synth.pack([c["src"] for c in cases])
    return cases, buf, lex_oracle.lex_batch(buf, off)


def test_golden_token_streams(oracle_run):
    cases, buf, (st, kl, ln, tto, status) = oracle_run
    assert len(cases) > 500
    n_tok = 0
    for i, c in enumerate(cases):
        if "raises" in c:
            assert status[i] == RAISE_CODE[c["raises"]], c["src"]
            continue
        assert status[i] == 0, c["src"]
        got = lex_oracle.as_reference_tokens(buf, st, kl, ln, int(tto[i]), int(tto[i + 1]))
        want = [tuple(t) for t in c["tokens"]]
        assert got == want, repr(c["src"][:200])
        n_tok += len(want)
    assert n_tok > 10000


def test_empty_batch_and_empty_tus():
    st, kl, ln, tto, status = lex_oracle.lex_batch(b"", np.array([0, 0, 0], np.uint64))
    assert list(tto) == [0, 1, 2]
    assert [int(k) >> 24 for k in kl] == [88, 88]
    assert list(ln) == [1, 1]
