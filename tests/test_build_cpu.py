"""The in-tree build's staleness rule: an object is as new as the moment its
compile started, so a source or header edited while nvcc ran (or after)
makes it stale."""
import os
import time

from opencuda import build


def test_object_stale_after_an_edit_during_compile(tmp_path):
    src = tmp_path / "k.cu"
    hdr = tmp_path / "k.cuh"
    obj = tmp_path / "k.o"
    dep = tmp_path / "k.d"
    for f in (src, hdr, obj):
        f.write_text("x")
    dep.write_text(f"{obj}: {src} \\\n {hdr}\n")
    t0 = time.time() - 100
    os.utime(src, (t0 - 10, t0 - 10))
    os.utime(hdr, (t0 - 10, t0 - 10))
    os.utime(obj, (t0, t0))              # the compile started at t0
    assert not build._obj_stale(src, obj, dep)
    os.utime(hdr, (t0 + 5, t0 + 5))      # header edited while nvcc ran
    assert build._obj_stale(src, obj, dep)
    os.utime(hdr, (t0 - 10, t0 - 10))
    dep.unlink()
    assert build._obj_stale(src, obj, dep)   # no dependency file: rebuild

