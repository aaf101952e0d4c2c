"""Host-side fault handling of ``compile_batch`` across devices, on CPU: the
failure is injected on the host (a stand-in for the per-device compile call
that raises, as a CUDA error or the library's watchdog would), never on a
GPU.  The failed device's TUs are split again over the devices that
succeeded and every result comes back in input order."""
import threading

import numpy as np
import pytest

from opencuda import api, compiler


def _fake(fail_devices, calls):
    lock = threading.Lock()

    def compile_on(device, slot, blobs, arch):
        with lock:
            calls.append((device, len(blobs)))
        if device in fail_devices:
            raise api.OcbError(f"device {device}: watchdog: stream made no progress")
        texts = [b"PTX:" + b for b in blobs]
        off = np.zeros(len(texts) + 1, np.uint64)
        np.cumsum([len(t) for t in texts], out=off[1:])
        return b"".join(texts), off, np.zeros(len(texts), np.int32)
    return compile_on


def test_failed_device_share_is_requeued(monkeypatch):
    calls = []
    monkeypatch.setattr(compiler, "_compile_on", _fake({1}, calls))
    srcs = [f"k{i}" * (i + 1) for i in range(40)]
    res = compiler.compile_batch(srcs, devices=[0, 1, 2])
    assert [r.ptx for r in res] == ["PTX:" + s for s in srcs]
    assert all(r.ok for r in res)
    first = [d for d, _ in calls[:3]]
    assert sorted(first) == [0, 1, 2]
    # the second round only uses the devices that succeeded
    assert {d for d, _ in calls[3:]} <= {0, 2} and len(calls) > 3


def test_every_device_failing_raises(monkeypatch):
    monkeypatch.setattr(compiler, "_compile_on", _fake({0, 1}, []))
    with pytest.raises(api.OcbError, match="watchdog"):
        compiler.compile_batch(["a", "b", "c"], devices=[0, 1])
