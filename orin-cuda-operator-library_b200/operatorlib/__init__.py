"""B200 (sm_100a) operator library: Python host side.

Two ways in, both onto the same compiled kernels in ``libopl_b200.so``:

* ``load_operatorlib()`` registers ``torch.ops.operatorlib.{reduce_sum,
  softmax, transpose, rmsnorm, gemm, attention}`` -- the same schemas as the
  reference's TORCH_LIBRARY binding (python/operatorlib_binding.cpp:190-206)
  and the same loader name as its python/load_extension.py:17.
* ``capi()`` returns the C-ABI (include/operatorlib/opl_capi.h) bound with
  ctypes; the raw-pointer helpers below call it with torch tensors' device
  pointers and the current stream, without going through the torch binding.

There is no CPU fallback: if the compiled library is missing, loading raises.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
LIB_PATH = PKG_DIR / "libopl_b200.so"
TORCH_LIB_PATH = PKG_DIR / "_operatorlib_torch.so"

_lock = threading.Lock()
_capi = None
_torch_loaded = False

CUDA_SUCCESS = 0
CUDA_ERROR_INVALID_VALUE = 1


class OplError(RuntimeError):
    """A C-ABI call returned a non-zero cudaError_t."""

    def __init__(self, op: str, code: int, text: str):
        super().__init__(f"{op} launch failed: {text} (cudaError {code})")
        self.code = code


def _bind(lib: ctypes.CDLL) -> ctypes.CDLL:
    vp, i, sz, f = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t, ctypes.c_float
    sigs = {
        "opl_reduce_sum_f32": [vp, vp, sz, vp],
        "opl_reduce_sum_partial_f64": [vp, vp, sz, vp],
        "opl_reduce_sum_f32_noalloc": [vp, vp, sz, vp],
        "opl_softmax_f32": [vp, vp, i, i, vp],
        "opl_softmax_f16": [vp, vp, i, i, vp],
        "opl_softmax_bf16": [vp, vp, i, i, vp],
        "opl_rmsnorm_f16": [vp, vp, vp, i, i, f, vp],
        "opl_rmsnorm_bf16": [vp, vp, vp, i, i, f, vp],
        "opl_transpose_f32": [vp, vp, i, i, vp],
        "opl_rmsnorm_f32": [vp, vp, vp, i, i, f, vp],
        "opl_gemm_f32": [vp, vp, vp, i, i, i, vp],
        "opl_gemm_f16": [vp, vp, vp, i, i, i, vp],
        "opl_attention_f32": [vp, vp, vp, vp, i, i, i, i, i, vp],
        "opl_attention_f16": [vp, vp, vp, vp, i, i, i, i, i, vp],
        "opl_read_and_clear_watchdog": [ctypes.POINTER(ctypes.c_int)],
    }
    for name, args in sigs.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = ctypes.c_int
    lib.opl_team_create.argtypes = [i, i, ctypes.POINTER(vp), ctypes.c_char_p]
    lib.opl_team_create.restype = ctypes.c_int
    lib.opl_team_connect.argtypes = [vp, ctypes.c_char_p]
    lib.opl_team_connect.restype = ctypes.c_int
    lib.opl_team_reduce_sum_f32.argtypes = [vp, vp, vp, sz, vp]
    lib.opl_team_reduce_sum_f32.restype = ctypes.c_int
    lib.opl_team_destroy.argtypes = [vp]
    lib.opl_team_destroy.restype = ctypes.c_int
    lib.opl_error_string.argtypes = [ctypes.c_int]
    lib.opl_error_string.restype = ctypes.c_char_p
    lib.opl_version.argtypes = []
    lib.opl_version.restype = ctypes.c_char_p
    return lib


def capi() -> ctypes.CDLL:
    """The C-ABI of libopl_b200.so (loaded once; raises if not built)."""
    global _capi
    with _lock:
        if _capi is None:
            if not LIB_PATH.exists():
                raise ImportError(
                    f"{LIB_PATH} is missing: build it with "
                    "orin-cuda-operator-library_b200/build.py (no CPU fallback)")
            _capi = _bind(ctypes.CDLL(str(LIB_PATH)))
    return _capi


def load_operatorlib(verbose: bool = False) -> None:
    """Registers torch.ops.operatorlib.* (CUDA dispatch key only)."""
    global _torch_loaded
    import torch

    with _lock:
        if _torch_loaded:
            return
        if not TORCH_LIB_PATH.exists():
            raise ImportError(f"{TORCH_LIB_PATH} is missing: run build.py")
        torch.ops.load_library(str(TORCH_LIB_PATH))
        _torch_loaded = True
    if verbose:
        print(f"operatorlib loaded from {TORCH_LIB_PATH}")


def check(op: str, code: int) -> None:
    if code != CUDA_SUCCESS:
        raise OplError(op, code, capi().opl_error_string(code).decode())


def version() -> str:
    return capi().opl_version().decode()


from .raw import (  # noqa: E402  (re-exported convenience layer)
    attention_into,
    gemm_into,
    reduce_sum_into,
    reduce_sum_partial_f64_into,
    rmsnorm_into,
    softmax_into,
    transpose_into,
)

from .team import ReduceTeam  # noqa: E402

__all__ = [
    "ReduceTeam",
    "OplError", "capi", "load_operatorlib", "check", "version",
    "attention_into", "gemm_into", "reduce_sum_into",
    "reduce_sum_partial_f64_into", "rmsnorm_into", "softmax_into",
    "transpose_into",
]
