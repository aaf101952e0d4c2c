"""The drop-in surface on the GPU: ``compile()``, ``compile_batch()`` and the
CLI ``python -m opencuda X.cu --emit-ptx`` against the reference's own
CLI ``python -m opencuda X.cu --emit-ptx`` (``opencuda/__main__.py:13-102``),
run unmodified from oracle/_ref/py: same file bytes, same stdout lines."""
import os
import subprocess
import sys
from pathlib import Path

import pytest

from oracle import ref_runner
from opencuda import compiler, synth
from tests._helpers import golden

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent


def _project(tmp: Path):
    """Sources that use quoted includes from an -I directory and from their
    own directory, plus an angle-bracket include."""
    inc = tmp / "inc"
    src = tmp / "src"
    inc.mkdir()
    src.mkdir()
    (inc / "tile.h").write_text("#define TILE 16\n#include \"scale.h\"\n")
    (inc / "scale.h").write_text("#define SCALE(x) ((x) * 2.0f)\n")
    (src / "util.h").write_text("#include \"tile.h\"\n#define N_ITER 4\n")
    sgemm = synth.SGEMM_SRC.replace("#define TILE 16", '#include <cuda_runtime.h>\n#include "tile.h"')
    assert sgemm != synth.SGEMM_SRC
    files = {
        "sgemm.cu": sgemm,
        "loop.cu": ('#include "util.h"\n'
                    "__global__ void loop(float *x, int n) {\n"
                    "    int i = blockIdx.x * blockDim.x + threadIdx.x;\n"
                    "    float acc = 0.0f;\n"
                    "    for (int k = 0; k < N_ITER; k++) { acc = acc + SCALE(x[i + k]); }\n"
                    "    if (i < n) x[i] = acc * TILE;\n"
                    "}\n"),
        "rand0.cu": synth.random_kernel(77, 0),
        "two.cu": ("__global__ void a(int *p) { p[0] = 1; }\n"
                   "__global__ void b(float *q, float s) { q[threadIdx.x] = s * 3.0f; }\n"),
    }
    for nm, text in files.items():
        (src / nm).write_text(text)
    return inc, src, list(files)


def _ours(args, cwd):
    env = dict(os.environ, PYTHONPATH=str(ROOT))
    return subprocess.run([sys.executable, "-m", "opencuda", *map(str, args)], cwd=cwd,
                          env=env, capture_output=True, text=True, timeout=600)


@pytest.mark.parametrize("arch", [None, "sm_89"])
def test_cli_file_bytes_and_stdout_match_reference_cli(tmp_path, arch):
    inc, src, names = _project(tmp_path)
    extra = ["--arch", arch] if arch else []
    for nm in names:
        f = src / nm
        rc, out, err = ref_runner.run_cli([f, "--emit-ptx", "--out", tmp_path / "ref.ptx",
                                           "-I", inc, *extra], cwd=tmp_path)
        assert rc == 0, err
        p = _ours([f, "--emit-ptx", "--out", tmp_path / "ours.ptx", "-I", inc, *extra],
                  cwd=tmp_path)
        assert p.returncode == 0, p.stderr
        assert (tmp_path / "ours.ptx").read_bytes() == (tmp_path / "ref.ptx").read_bytes(), nm
        ref_lines = [ln.replace(str(tmp_path / "ref.ptx"), "OUT") for ln in out.splitlines()]
        our_lines = [ln.replace(str(tmp_path / "ours.ptx"), "OUT") for ln in p.stdout.splitlines()]
        assert our_lines == ref_lines


def test_cli_batch_writes_every_file(tmp_path):
    inc, src, names = _project(tmp_path)
    files = [src / nm for nm in names]
    p = _ours([*files, "--emit-ptx", "-I", inc], cwd=tmp_path)
    assert p.returncode == 0, p.stderr
    for f in files:
        rc, _, err = ref_runner.run_cli([f, "--emit-ptx", "--out", tmp_path / "ref.ptx",
                                         "-I", inc], cwd=tmp_path)
        assert rc == 0, err
        assert f.with_suffix(".ptx").read_bytes() == (tmp_path / "ref.ptx").read_bytes()


def test_cli_reports_reference_error_and_exits_1(tmp_path):
    case = next(c for c in golden("ir_golden.json.gz")["cases"]
                if c.get("raises") == "ParseError")
    f = tmp_path / "bad.cu"
    f.write_text(case["src"])
    rc, _, _ = ref_runner.run_cli([f, "--emit-ptx"], cwd=tmp_path)
    assert rc == 1
    p = _ours([f, "--emit-ptx"], cwd=tmp_path)
    assert p.returncode == 1 and "ParseError" in p.stderr
    assert not f.with_suffix(".ptx").exists()


def test_compile_and_compile_error():
    with ref_runner.RefPool(2) as pool:
        want = pool.run([synth.SGEMM_SRC], what=("ptx",))
        want89 = pool.run([synth.SGEMM_SRC], what=("ptx",), arch="sm_89")
    assert compiler.compile(synth.SGEMM_SRC) == want[0]["ptx"]
    assert compiler.compile(synth.SGEMM_SRC, arch="sm_89") == want89[0]["ptx"]
    case = next(c for c in golden("ir_golden.json.gz")["cases"]
                if c.get("raises") == "ParseError")
    with pytest.raises(compiler.CompileError) as ei:
        compiler.compile(case["src"])
    assert ei.value.exc_type == "ParseError" and ei.value.status == 3


def test_compile_batch_sharded_slots_keep_input_order():
    import torch
    srcs = synth.random_batch(96, seed=404) + [synth.SGEMM_SRC, ""]
    one = compiler.compile_batch(srcs)
    devs = [0, 0, 0] if torch.cuda.device_count() < 2 else list(range(torch.cuda.device_count()))
    many = compiler.compile_batch(srcs, devices=devs)
    assert [(r.status, r.ptx) for r in many] == [(r.status, r.ptx) for r in one]
    with ref_runner.RefPool() as pool:
        ref = pool.run(srcs, what=("ptx",), chunksize=4)
    for r, w in zip(one, ref):
        if "ptx" in w:
            assert r.ok and r.ptx == w["ptx"]
        else:
            assert not r.ok
