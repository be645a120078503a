"""The reference's own tests, run unchanged against this library.

* Its three launcher smoke tests (tests/core_ops_smoke.cu, gemm_smoke.cu,
  attention_smoke.cu), compiled from a reference checkout and linked against
  this library's static archive (oracle/build_oracle.py,
  build_reference_smoke; gemm_smoke uses cuBLAS as its oracle, as in the
  reference) -- the drop-in check for C++ callers of
  include/operatorlib/operators.h.
* Its PyTorch extension test (python/test_extension.py, main()), staged
  unchanged next to those binaries and run with this package's
  load_extension.py on PYTHONPATH -- the drop-in check for Python callers of
  torch.ops.operatorlib.
* This library's own launcher smoke test (tests/cpp/operators_smoke.cu),
  built by the package's build.py against the same archive.
Each must exit 0 and print its PASS lines.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

REPO = Path(__file__).resolve().parents[1]
SMOKE = REPO / "oracle" / "_ref" / "smoke"
OWN = REPO / "orin-cuda-operator-library_b200" / "_build" / "bin" / "operatorlib_b200_smoke"
PY_DIR = REPO / "orin-cuda-operator-library_b200" / "python"

EXPECT = {
    "core_ops_smoke": ["reduce_sum_f32=PASS", "transpose_f32=PASS", "core_ops_smoke=PASS"],
    "gemm_smoke": ["gemm_smoke=PASS"],
    "attention_smoke": ["attention_smoke=PASS"],
}


def _run(cmd, **kw):
    return subprocess.run(cmd, capture_output=True, text=True, timeout=600, **kw)


def test_own_launcher_smoke(cuda):
    if not OWN.exists():
        pytest.fail(f"{OWN} not built (run the package build.py)")
    proc = _run([str(OWN)])
    assert proc.returncode == 0, proc.stdout + proc.stderr
    assert "operatorlib_b200_smoke=PASS" in proc.stdout


@pytest.mark.parametrize("name", sorted(EXPECT))
def test_reference_launcher_smoke(cuda, name):
    exe = SMOKE / name
    if not exe.exists():
        pytest.skip("reference smoke tests not built (no reference checkout at build time)")
    proc = _run([str(exe)])
    assert proc.returncode == 0, proc.stdout + proc.stderr
    assert "PASS" in proc.stdout and "FAIL" not in proc.stdout, proc.stdout
    for line in EXPECT[name]:
        assert line in proc.stdout


def test_reference_extension_test(cuda):
    script = SMOKE / "test_extension.py"
    if not script.exists():
        pytest.skip("reference test_extension.py not staged (no reference checkout at build time)")
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join([str(PY_DIR), env.get("PYTHONPATH", "")])
    proc = _run([sys.executable, str(script)], env=env, cwd=str(SMOKE))
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    assert "operatorlib_extension=PASS" in proc.stdout
