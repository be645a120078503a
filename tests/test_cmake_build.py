"""The CMake build (CMakeLists.txt at the repository root) configures and
builds the static library target `operatorlib` for sm_100a, exports the
reference's eight C++ launchers from it, and links the launcher smoke
test(s) against it -- on the CPU (nvcc cross-compiles; nothing is run)."""
from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
LAUNCHERS = ["reduce_sum_f32", "softmax_f32", "transpose_f32", "rmsnorm_f32", "gemm_f32",
             "gemm_f16", "attention_f32", "attention_f16"]


def _reference_tests_dir():
    root = os.environ.get("OPL_REFERENCE_ROOT")
    cand = Path(root) if root else REPO.parent / "reference"
    return cand / "tests" if (cand / "tests" / "core_ops_smoke.cu").exists() else None


@pytest.mark.skipif(shutil.which("cmake") is None, reason="cmake not installed")
def test_cmake_static_library(tmp_path):
    build = tmp_path / "build"
    args = ["cmake", "-S", str(REPO), "-B", str(build), "-DCMAKE_BUILD_TYPE=Release",
            "-G", "Ninja" if shutil.which("ninja") else "Unix Makefiles"]
    ref_tests = _reference_tests_dir()
    if ref_tests is not None:
        args.append(f"-DOPERATORLIB_REFERENCE_TESTS={ref_tests}")
    proc = subprocess.run(args, capture_output=True, text=True, timeout=300)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    proc = subprocess.run(["cmake", "--build", str(build), "-j", str(os.cpu_count() or 4)],
                          capture_output=True, text=True, timeout=1200)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    archive = build / "liboperatorlib.a"
    assert archive.exists()
    syms = subprocess.run(["nm", "-C", "--defined-only", str(archive)], capture_output=True,
                          text=True).stdout
    for name in LAUNCHERS:
        assert f"operatorlib::{name}(" in syms, name
    assert (build / "operatorlib_b200_smoke").exists()
    if ref_tests is not None:
        for exe in ("operatorlib_core_smoke", "operatorlib_gemm_smoke",
                    "operatorlib_attention_smoke"):
            assert (build / exe).exists(), exe
    listing = subprocess.run(["ctest", "--test-dir", str(build), "-N"], capture_output=True,
                             text=True).stdout
    assert "operatorlib_b200_smoke" in listing
