"""The allocation-free lexer entry point (ocb_lex_device_static).

It exists for callers that may not allocate device memory when they lex --
code inside another framework's memory pool or a fixed arena that forbids
cudaMalloc/cudaFree after start-up -- so its scratch is one fixed array in the
library.  These tests call it through the C ABI twice in a row, on two
different batches, and require output identical (bit-exact, as every lexer
test here) to the context-based ocb_lex_device; the first batch makes the
reference raise on some TUs and the second does not, so leftovers of the first
call in the shared array would show up in the second.  This file is collected
last so that a stop-at-first-failure run has run everything else before it.
"""
import ctypes

import numpy as np
import pytest

from opencuda import _lib, synth
from opencuda.api import pack_sources
from tests._helpers import fuzz_sources

pytestmark = pytest.mark.gpu


def _device_batch(torch, srcs, dev):
    buf, off = pack_sources(srcs)
    n_tu = len(srcs)
    cap = len(buf) + n_tu + 1
    d = {
        "src": torch.from_numpy(buf.copy()).to(dev),
        "off": torch.from_numpy(off.view(np.int64).copy()).to(dev),
        "n_bytes": len(buf), "n_tu": n_tu, "cap": cap,
    }
    return d


def _outputs(torch, d, dev):
    return {k: torch.full((n,), -7, dtype=dt, device=dev) for k, n, dt in (
        ("start", d["cap"], torch.int32), ("kl", d["cap"], torch.int32),
        ("line", d["cap"], torch.int32), ("tto", d["n_tu"] + 1, torch.int64),
        ("status", d["n_tu"], torch.int32), ("n", 1, torch.int64))}


def _host(o):
    n = int(o["n"].item())
    return {"n": n,
            "start": o["start"][:n].cpu().numpy(), "kl": o["kl"][:n].cpu().numpy(),
            "line": o["line"][:n].cpu().numpy(), "tto": o["tto"].cpu().numpy(),
            "status": o["status"].cpu().numpy()}


def _run_existing(ctx, torch, d, dev, stream):
    o = _outputs(torch, d, dev)
    ctx.lex_device(d["src"].data_ptr(), d["n_bytes"], d["off"].data_ptr(), d["n_tu"],
                   o["start"].data_ptr(), o["kl"].data_ptr(), o["line"].data_ptr(), d["cap"],
                   o["tto"].data_ptr(), o["status"].data_ptr(), o["n"].data_ptr(),
                   stream.cuda_stream)
    torch.cuda.synchronize()
    return _host(o)


def _run_static(lib, torch, d, dev, stream):
    o = _outputs(torch, d, dev)
    err = ctypes.create_string_buffer(256)
    rc = lib.ocb_lex_device_static(
        d["src"].data_ptr(), d["n_bytes"], d["off"].data_ptr(), d["n_tu"],
        o["start"].data_ptr(), o["kl"].data_ptr(), o["line"].data_ptr(), d["cap"],
        o["tto"].data_ptr(), o["status"].data_ptr(), o["n"].data_ptr(),
        stream.cuda_stream, err, len(err))
    assert rc == 0, err.value.decode()
    torch.cuda.synchronize()
    return _host(o)


def test_static_entry_point_matches_existing_two_calls_in_a_row(ctx):
    import torch
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)
    lib = _lib.load()
    # batch A: fuzz with raising hex floats, empty TUs and unterminated text
    a_srcs = fuzz_sources(3000, 42) + ["", "0x.p1", "0x1p1024", '"open', "/* open"]
    # batch B: larger, different sizes, nothing raises
    b_srcs = [synth.SGEMM_SRC] + synth.random_batch(600, seed=9)
    batches = [_device_batch(torch, a_srcs, dev), _device_batch(torch, b_srcs, dev)]
    assert all(b["n_bytes"] <= 4 << 20 and b["n_tu"] <= 16384 for b in batches)
    expected = [_run_existing(ctx, torch, b, dev, stream) for b in batches]
    assert (expected[0]["status"] != 0).any() and not (expected[1]["status"] != 0).any()
    for b, want in zip(batches, expected):       # two calls in a row
        got = _run_static(lib, torch, b, dev, stream)
        assert got["n"] == want["n"]
        for key in ("start", "kl", "line", "tto", "status"):
            assert np.array_equal(got[key], want[key]), key


def test_static_entry_point_rejects_oversized_batches():
    import torch
    dev = torch.device("cuda:0")
    lib = _lib.load()
    small = torch.zeros(64, dtype=torch.uint8, device=dev)
    off = torch.zeros(2, dtype=torch.int64, device=dev)
    err = ctypes.create_string_buffer(256)
    rc = lib.ocb_lex_device_static(small.data_ptr(), (4 << 20) + 1, off.data_ptr(), 1,
                                   None, None, None, 0, None, None, None, None,
                                   err, len(err))
    assert rc == -2 and b"4 MiB" in err.value
    rc = lib.ocb_lex_device_static(small.data_ptr(), 16, off.data_ptr(), 16385,
                                   None, None, None, 0, None, None, None, None,
                                   err, len(err))
    assert rc == -2 and b"16384" in err.value
