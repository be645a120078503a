"""Build recipe for the CPU oracle and the reference builds -- TEST INFRASTRUCTURE.

Outputs (all git-ignored build products; they travel with the tree):
  oracle/liboracle.so              gcc build of oracle/opl_oracle.c (always).
  oracle/_ref/libref_operatorlib.so  the reference's own launchers and kernels
                                   (its src/*.cu, unmodified, compiled in place
                                   for sm_100a) behind C entry points
                                   (ref_shim/ref_launchers_capi.cu).
  oracle/_ref/libref_cpu.so        the reference's own CPU verification loops,
                                   compiled from its standalone sources in
                                   place (ref_shim/ref_cpu_*.cu).
  oracle/_ref/smoke/               the reference's own launcher smoke tests
                                   (its tests/*_smoke.cu, unmodified) linked
                                   against THIS library's static archive, and
                                   a staged copy of its python/test_extension.py
                                   (run unchanged against this library's
                                   torch binding); checkers, never shipped.
The two _ref libraries are built only where the reference tree exists: the
directory named by --reference-root or OPL_REFERENCE_ROOT, else a checkout
named `reference` beside this repository's directory.  Elsewhere the
prebuilt copies are used as they are, silently.  No reference source is
copied: each file is compiled where it lies.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

ORACLE = Path(__file__).resolve().parent
REF_OUT = ORACLE / "_ref"
SHIM = ORACLE / "ref_shim"
NVCC = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
REF_CPU = {
    "reduce": "reduce/reduce_v3.cu",
    "softmax": "softmax/softmax_v4.cu",
    "transpose": "transpose/transpose_v2.cu",
    "rmsnorm": "rmsnorm/rmsnorm_v3.cu",
    "attention": "attention/attention_common.h",
}
REF_SRC = ["reduce.cu", "softmax.cu", "transpose.cu", "rmsnorm.cu", "gemm.cu",
           "attention.cu"]


def reference_root(explicit: str | None = None) -> Path | None:
    given = explicit or os.environ.get("OPL_REFERENCE_ROOT")
    root = Path(given) if given else ORACLE.parent.parent / "reference"
    return root if (root / "src" / "reduce.cu").exists() else None


def _run(cmd: list[str]) -> None:
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"failed: {' '.join(cmd)}\n{proc.stdout}\n{proc.stderr}")


def _newer(target: Path, deps: list[Path]) -> bool:
    return target.exists() and all(d.stat().st_mtime <= target.stat().st_mtime
                                   for d in deps)


def build_oracle() -> Path:
    src = ORACLE / "opl_oracle.c"
    lib = ORACLE / "liboracle.so"
    if not _newer(lib, [src]):
        _run(["gcc", "-O2", "-fPIC", "-shared", "-fno-fast-math", "-o", str(lib),
              str(src), "-lm"])
    return lib


def build_reference(reference: str | None = None) -> list[Path]:
    root = reference_root(reference)
    if root is None:
        return []
    REF_OUT.mkdir(exist_ok=True)
    built = []
    # Reference launchers + kernels.
    lib = REF_OUT / "libref_operatorlib.so"
    srcs = [root / "src" / s for s in REF_SRC] + [SHIM / "ref_launchers_capi.cu"]
    if not _newer(lib, srcs):
        objs = []
        for s in srcs:
            obj = REF_OUT / ("launch_" + s.stem + ".o")
            _run([NVCC, *ARCH, "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
                  f"-I{root / 'include'}", "-c", str(s), "-o", str(obj)])
            objs.append(obj)
        _run([NVCC, *ARCH, "-shared", "-cudart", "static", "-o", str(lib),
              *map(str, objs), "-Xlinker", "-Bsymbolic"])
    built.append(lib)
    # Reference CPU loops.
    lib = REF_OUT / "libref_cpu.so"
    shims = [SHIM / f"ref_cpu_{op}.cu" for op in REF_CPU]
    if not _newer(lib, shims + [root / p for p in REF_CPU.values()]):
        objs = []
        for op, rel in REF_CPU.items():
            obj = REF_OUT / f"cpu_{op}.o"
            _run([NVCC, *ARCH, "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
                  f'-DREF_SOURCE="{root / rel}"', f"-I{root / Path(rel).parent}",
                  "-c", str(SHIM / f"ref_cpu_{op}.cu"), "-o", str(obj)])
            objs.append(obj)
        _run([NVCC, *ARCH, "-shared", "-cudart", "static", "-o", str(lib),
              *map(str, objs), "-Xlinker", "-Bsymbolic"])
    built.append(lib)
    return built


REF_SMOKE = {"core_ops_smoke": [], "attention_smoke": [], "gemm_smoke": ["-lcublas"]}


def build_reference_smoke(reference: str | None = None) -> list[Path]:
    """The reference's C++ smoke tests built against this library (the
    package's liboperatorlib.a must exist: build it first)."""
    root = reference_root(reference)
    if root is None:
        return []
    import importlib.util
    import shutil

    spec = importlib.util.spec_from_file_location(
        "opl_build", ORACLE.parent / "orin-cuda-operator-library_b200" / "build.py")
    opl_build = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(opl_build)
    out_dir = REF_OUT / "smoke"
    built = [opl_build.link_against_archive(root / "tests" / f"{name}.cu", out_dir / name, extra)
             for name, extra in REF_SMOKE.items()]
    staged = out_dir / "test_extension.py"
    src = root / "python" / "test_extension.py"
    if not _newer(staged, [src]):
        shutil.copyfile(src, staged)
    built.append(staged)
    return built


def main(argv=None) -> int:
    import argparse

    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--reference-root", default=None,
                   help="reference checkout to compile oracle/_ref from")
    args = p.parse_args(argv)
    print(build_oracle())
    for p in build_reference(args.reference_root):
        print(p)
    for p in build_reference_smoke(args.reference_root):
        print(p)
    return 0


if __name__ == "__main__":
    sys.exit(main())
