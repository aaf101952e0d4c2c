"""GPU lexer parity: libocb's sm_100a lexer against the reference's token
streams (golden fixtures) and against the C oracle (oracle/lex_oracle.c) on
seeded inputs, through the C ABI."""
import os

import numpy as np
import pytest

from oracle import lex_oracle
from opencuda import synth
from opencuda.api import pack_sources
from tests._helpers import golden, RAISE_CODE, fuzz_sources

pytestmark = pytest.mark.gpu


def assert_same_as_oracle(tb, buf, off):
    st, kl, ln, tto, status = lex_oracle.lex_batch(buf, off)
    assert np.array_equal(tb.tu_tok_off, tto), "per-TU token offsets differ"
    assert np.array_equal(tb.status, status), "per-TU status differs"
    for name, a, b in (("start", tb.start, st), ("kindlen", tb.kindlen, kl),
                       ("line", tb.line, ln)):
        if not np.array_equal(a, b):
            n = min(len(a), len(b))
            d = np.flatnonzero(a[:n] != b[:n])
            raise AssertionError(f"{name} differs: n={len(a)} vs {len(b)}, first at {d[:5]}")


def test_golden_token_streams(ctx):
    cases = golden("lex_golden.json.gz")["cases"]
    tb = ctx.lex_batch([c["src"] for c in cases])
    for i, c in enumerate(cases):
        if "raises" in c:
            assert tb.status[i] == RAISE_CODE[c["raises"]], c["src"]
        else:
            assert tb.status[i] == 0
            assert tb.tokens(i) == [tuple(t) for t in c["tokens"]], repr(c["src"][:200])


@pytest.mark.parametrize("seed", [1, 2, 3])
def test_fuzz_matches_oracle(ctx, seed):
    srcs = fuzz_sources(6000, seed)
    buf, off = pack_sources(srcs)
    assert_same_as_oracle(ctx.lex_batch(buf=buf, tu_off=off), buf, off)


def test_tiny_and_empty_tus(ctx):
    srcs = ["", "", "a", "", "/", "", "'", '"x', "", "/*", "*/", ""] * 50 + [""]
    buf, off = pack_sources(srcs)
    assert_same_as_oracle(ctx.lex_batch(buf=buf, tu_off=off), buf, off)
    buf, off = pack_sources(["", "", ""])
    tb = ctx.lex_batch(buf=buf, tu_off=off)
    assert list(tb.tu_tok_off) == [0, 1, 2, 3] and list(tb.kind) == [88] * 3


def test_one_long_tu_crossing_many_tiles(ctx):
    # one TU much larger than a thread window / block tile, with a long string,
    # a long block comment and an unterminated string at the end
    body = ("int x = 1; /* " + "c" * 20000 + " */ s = \"" + "q" * 30000 + "\";\n") * 3
    srcs = [body + 'tail = 1; "never closed ' + "z" * 5000]
    buf, off = pack_sources(srcs)
    assert_same_as_oracle(ctx.lex_batch(buf=buf, tu_off=off), buf, off)


def test_workloads_match_oracle(ctx):
    buf, off = synth.lexstress_batch(total_bytes=16 << 20, tu_bytes=16384, seed=11,
                                     pool_lines=50_000)
    buf = np.frombuffer(buf, np.uint8)
    assert_same_as_oracle(ctx.lex_batch(buf=buf, tu_off=off), buf, off)
    srcs = [synth.SGEMM_SRC] + synth.random_batch(256, seed=5)
    buf, off = pack_sources(srcs)
    assert_same_as_oracle(ctx.lex_batch(buf=buf, tu_off=off), buf, off)


def test_full_size_against_oracle(ctx):
    """The whole 1 GiB stress text (65,536 TUs of 16 KiB): every token of
    every TU equals the oracle's, and lexing the batch equals lexing its four
    TU shards separately (positions re-based)."""
    from concurrent.futures import ThreadPoolExecutor
    buf, off = synth.lexstress_batch(total_bytes=1 << 30, tu_bytes=16384, seed=99)
    buf = np.frombuffer(buf, np.uint8)
    full = ctx.lex_batch(buf=buf, tu_off=off)
    n_tu = len(off) - 1
    cuts = [0, n_tu // 4, n_tu // 2, 3 * n_tu // 4, n_tu]
    for a, b in zip(cuts[:-1], cuts[1:]):
        base = int(off[a])
        sub_off = off[a:b + 1] - off[a]
        part = ctx.lex_batch(buf=buf[base:int(off[b])], tu_off=sub_off)
        t0, t1 = int(full.tu_tok_off[a]), int(full.tu_tok_off[b])
        assert np.array_equal(full.start[t0:t1] - np.uint32(base), part.start)
        assert np.array_equal(full.kindlen[t0:t1], part.kindlen)
        assert np.array_equal(full.line[t0:t1], part.line)
        assert np.array_equal(full.status[a:b], part.status)
        del part

    # the oracle over every TU, in chunks on all host cores (the C library
    # releases the GIL)
    def chunk(ab):
        a, b = ab
        base = int(off[a])
        sub = off[a:b + 1] - off[a]
        st, kl, ln, tto, status = lex_oracle.lex_batch(buf[base:int(off[b])], sub)
        t0, t1 = int(full.tu_tok_off[a]), int(full.tu_tok_off[b])
        return (np.array_equal(full.start[t0:t1] - np.uint32(base), st)
                and np.array_equal(full.kindlen[t0:t1], kl)
                and np.array_equal(full.line[t0:t1], ln)
                and np.array_equal(full.tu_tok_off[a:b + 1] - np.uint64(t0), tto)
                and np.array_equal(full.status[a:b], status))

    step = 512
    parts = [(a, min(n_tu, a + step)) for a in range(0, n_tu, step)]
    with ThreadPoolExecutor(max_workers=len(os.sched_getaffinity(0))) as ex:
        same = list(ex.map(chunk, parts))
    assert all(same), [p for p, ok in zip(parts, same) if not ok][:4]


def test_device_entry_point(ctx):
    """ocb_lex_device on torch-owned device buffers equals ocb_lex_batch."""
    import torch
    srcs = synth.random_batch(64, seed=3)
    buf, off = pack_sources(srcs)
    ref = ctx.lex_batch(buf=buf, tu_off=off)
    dev = torch.device("cuda:0")
    d_src = torch.from_numpy(buf.copy()).to(dev)
    d_off = torch.from_numpy(off.view(np.int64).copy()).to(dev)
    cap = len(buf) + len(srcs) + 1
    d_start = torch.empty(cap, dtype=torch.int32, device=dev)
    d_kl = torch.empty(cap, dtype=torch.int32, device=dev)
    d_line = torch.empty(cap, dtype=torch.int32, device=dev)
    d_tto = torch.empty(len(srcs) + 1, dtype=torch.int64, device=dev)
    d_status = torch.empty(len(srcs), dtype=torch.int32, device=dev)
    d_n = torch.zeros(1, dtype=torch.int64, device=dev)
    stream = torch.cuda.current_stream(dev)
    ctx.lex_device(d_src.data_ptr(), len(buf), d_off.data_ptr(), len(srcs), d_start.data_ptr(),
                   d_kl.data_ptr(), d_line.data_ptr(), cap, d_tto.data_ptr(),
                   d_status.data_ptr(), d_n.data_ptr(), stream.cuda_stream)
    torch.cuda.synchronize()
    n = int(d_n.item())
    assert n == len(ref.start)
    assert np.array_equal(d_start[:n].cpu().numpy().view(np.uint32), ref.start)
    assert np.array_equal(d_kl[:n].cpu().numpy().view(np.uint32), ref.kindlen)
    assert np.array_equal(d_line[:n].cpu().numpy().view(np.uint32), ref.line)
    assert np.array_equal(d_tto.cpu().numpy().view(np.uint64), ref.tu_tok_off)


def _fused(ctx, buf, off):
    """ocb_lex_device without the line array: the single-pass lexer."""
    import torch
    dev = torch.device("cuda:0")
    n_tu = len(off) - 1
    d_src = torch.from_numpy(np.ascontiguousarray(buf, np.uint8).copy() if len(buf)
                             else np.zeros(16, np.uint8)).to(dev)
    d_off = torch.from_numpy(np.asarray(off, np.uint64).view(np.int64).copy()).to(dev)
    cap = len(buf) + n_tu + 1
    d_start = torch.empty(cap, dtype=torch.int32, device=dev)
    d_kl = torch.empty(cap, dtype=torch.int32, device=dev)
    d_tto = torch.empty(n_tu + 1, dtype=torch.int64, device=dev)
    d_status = torch.empty(max(n_tu, 1), dtype=torch.int32, device=dev)
    d_n = torch.zeros(1, dtype=torch.int64, device=dev)
    stream = torch.cuda.current_stream(dev)
    ctx.lex_device(d_src.data_ptr(), len(buf), d_off.data_ptr(), n_tu, d_start.data_ptr(),
                   d_kl.data_ptr(), 0, cap, d_tto.data_ptr(), d_status.data_ptr(),
                   d_n.data_ptr(), stream.cuda_stream)
    torch.cuda.synchronize()
    n = int(d_n.item())
    return (d_start[:n].cpu().numpy().view(np.uint32), d_kl[:n].cpu().numpy().view(np.uint32),
            d_tto.cpu().numpy().view(np.uint64), d_status[:n_tu].cpu().numpy())


def _edge_batches():
    """TU layouts and texts the single-pass lexer's tiles must get right:
    empty TUs at the start, middle and end, one-byte TUs, a comment and a
    string far longer than a tile, runs of tokens with no whitespace (more
    records than a thread buffers), unterminated comments and strings, hex
    floats the reference rejects, CRLF text, and TUs cut mid-token."""
    long_run = "+".join(f"v{i}" for i in range(6000))
    yield ["", "", "a b", "", "x"]
    yield ["x"] * 3000
    yield ["", "/*" + "c" * 40000 + "*/ int a;", "", '"' + "s" * 30000 + '" b', ""]
    yield [long_run, "y" + long_run, "// " + "q" * 20000 + "\nz = 1;"]
    yield ["a /* open", '"open', "'x", "0x1.p4 0x.p1 0x1p99999 1.5e3f", "a\r\nb\r\n"]
    yield ["int a;\n" * 3000, "\n" * 9000, " " * 9000 + "k"]
    rnd = fuzz_sources(400, 21)
    yield rnd
    yield [s[: len(s) // 2] for s in rnd]


def test_single_pass_equals_multi_pass(ctx):
    """The single-pass lexer (no per-token lines) gives the same token
    records, per-TU offsets and statuses as the multi-pass pipeline, which
    the other tests pin to the oracle."""
    batches = list(_edge_batches())
    buf, off = synth.lexstress_batch(total_bytes=24 << 20, tu_bytes=16384, seed=17,
                                     pool_lines=50_000)
    big = [buf[int(off[i]):int(off[i + 1])].decode() for i in range(len(off) - 1)]
    batches.append(big)
    batches.append([synth.SGEMM_SRC] + synth.random_batch(300, seed=9) + [""])
    for srcs in batches:
        b, o = pack_sources(srcs)
        ref = ctx.lex_batch(buf=b, tu_off=o)
        st, kl, tto, status = _fused(ctx, b, o)
        assert np.array_equal(status, ref.status)
        assert np.array_equal(tto, ref.tu_tok_off)
        assert np.array_equal(st, ref.start)
        assert np.array_equal(kl, ref.kindlen)
