"""In-tree build of the B200 operator library (sm_100a only).

Produces, next to the Python package ``operatorlib``:
  * ``libopl_b200.so``       -- every CUDA kernel, the C-ABI (opl_*) and the
                                C++ API of include/operatorlib/operators.h;
  * ``_operatorlib_torch.so`` -- the TORCH_LIBRARY(operatorlib, ...) binding,
                                linked against libopl_b200.so;
  * ``liboperatorlib.a``      -- the same objects as a static archive, the
                                counterpart of the reference's static library
                                target (CMakeLists.txt at the repository root
                                builds the same archive through CMake);
  * ``_build/bin/operatorlib_b200_smoke`` -- tests/cpp/operators_smoke.cu
                                linked against that archive.

This replaces the reference's CMake static library (CMakeLists.txt:16-36,
CUDA_ARCHITECTURES 87) and JIT loader (python/load_extension.py:17-36): nvcc
and g++ are driven directly so the built objects live in the tree and travel
with it.  Objects are rebuilt only when a source or header is newer.

Usage: python orin-cuda-operator-library_b200/build.py [--force] [-j N]
"""
from __future__ import annotations

import argparse
import concurrent.futures as futures
import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent
REPO = PKG_ROOT.parent
CSRC = PKG_ROOT / "csrc"
INCLUDE = REPO / "include"
OUT_DIR = PKG_ROOT / "operatorlib"
OBJ_DIR = PKG_ROOT / "_build"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
    "--expt-relaxed-constexpr",
    "-DOPL_BUILDING_LIBRARY",
]
LIB_NAME = "libopl_b200.so"
STATIC_NAME = "liboperatorlib.a"
BIN_DIR = OBJ_DIR / "bin"
TORCH_LIB_NAME = "_operatorlib_torch.so"


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.rglob("*.h"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _run(cmd: list[str]) -> None:
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(
            f"command failed ({proc.returncode}): {' '.join(cmd)}\n"
            f"{proc.stdout}\n{proc.stderr}")


def _compile_cu(src: Path, force: bool) -> Path:
    obj = OBJ_DIR / (src.stem + ".o")
    if force or _stale(obj, [src] + _headers()):
        _run([NVCC, *NVCC_FLAGS, f"-I{INCLUDE}", f"-I{CSRC}", "-c", str(src),
              "-o", str(obj)])
    return obj


def build_library(force: bool = False, jobs: int = 8) -> Path:
    OBJ_DIR.mkdir(exist_ok=True)
    OUT_DIR.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    with futures.ThreadPoolExecutor(max_workers=jobs) as pool:
        objects = list(pool.map(lambda s: _compile_cu(s, force), sources))
    lib = OUT_DIR / LIB_NAME
    if force or _stale(lib, objects):
        # Static cudart: the library carries its own runtime and needs no
        # LD_LIBRARY_PATH; device pointers and streams from any other runtime
        # in the process (e.g. torch's) share the device's primary context.
        _run([NVCC, *ARCH, "-shared", "-cudart", "static", "-o", str(lib),
              *map(str, objects), "-Xlinker", "--no-undefined", "-lpthread",
              "-ldl", "-lrt"])
    archive = OUT_DIR / STATIC_NAME
    if force or _stale(archive, objects):
        if archive.exists():
            archive.unlink()
        _run(["ar", "rcs", str(archive), *map(str, objects)])
    return lib


def link_against_archive(src: Path, out: Path, extra: list[str] | None = None,
                         force: bool = False) -> Path:
    """Compiles a C++/CUDA test program that includes operatorlib/operators.h
    and links it against the static archive (the way a CMake consumer of the
    `operatorlib` target links)."""
    archive = OUT_DIR / STATIC_NAME
    if force or _stale(out, [src, archive]):
        out.parent.mkdir(parents=True, exist_ok=True)
        _run([NVCC, *ARCH, "-O2", "-std=c++17", f"-I{INCLUDE}", str(src), "-o", str(out),
              str(archive), *(extra or [])])
    return out


def build_torch_binding(force: bool = False) -> Path:
    import torch
    from torch.utils import cpp_extension

    src = PKG_ROOT / "python" / "operatorlib_binding.cpp"
    lib = OUT_DIR / TORCH_LIB_NAME
    if not (force or _stale(lib, [src, OUT_DIR / LIB_NAME] + _headers())):
        return lib
    includes = cpp_extension.include_paths(device_type="cuda")
    lib_dirs = cpp_extension.library_paths(device_type="cuda")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O3", "-std=c++17", "-shared", "-fPIC",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_EXTENSION_NAME=_operatorlib_torch",
           f"-I{INCLUDE}", f"-I{CUDA_HOME / 'include'}",
           f"-I{sysconfig.get_paths()['include']}"]
    cmd += [f"-I{p}" for p in includes]
    cmd += [str(src), "-o", str(lib)]
    cmd += [f"-L{p}" for p in lib_dirs]
    cmd += [f"-Wl,-rpath,{p}" for p in lib_dirs]
    cmd += [f"-L{OUT_DIR}", "-l:" + LIB_NAME, "-Wl,-rpath,$ORIGIN",
            "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda"]
    _run(cmd)
    return lib


def build(force: bool = False, jobs: int = 8, torch_binding: bool = True) -> None:
    if shutil.which(NVCC) is None and not Path(NVCC).exists():
        raise RuntimeError(f"nvcc not found at {NVCC}")
    build_library(force=force, jobs=jobs)
    link_against_archive(REPO / "tests" / "cpp" / "operators_smoke.cu",
                         BIN_DIR / "operatorlib_b200_smoke", force=force)
    if torch_binding:
        build_torch_binding(force=force)


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--force", action="store_true")
    parser.add_argument("-j", "--jobs", type=int, default=os.cpu_count() or 4)
    parser.add_argument("--no-torch", action="store_true")
    args = parser.parse_args()
    build(force=args.force, jobs=args.jobs, torch_binding=not args.no_torch)
    print(f"built {OUT_DIR / LIB_NAME}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
