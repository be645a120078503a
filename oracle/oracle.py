"""Python handle on the CPU oracle -- TEST INFRASTRUCTURE ONLY.

Wraps oracle/liboracle.so (the C restatement, opl_oracle.c) and, when built,
oracle/_ref/libref_cpu.so (the reference's own CPU loops compiled from its
sources) with numpy-in / numpy-out functions.  Only tests/, the smoke check of
__graft_entry__ and bench.py's CPU-baseline legs use this module; the library
never does.
"""
from __future__ import annotations

import ctypes
import os
import threading
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
_LIB = None
_REF_CPU = None
_REF_GPU = None
_LOCK = threading.Lock()

_F = ctypes.POINTER(ctypes.c_float)
_D = ctypes.POINTER(ctypes.c_double)


def _fp(a: np.ndarray):
    return a.ctypes.data_as(_F)


def _dp(a: np.ndarray):
    return a.ctypes.data_as(_D)


def lib() -> ctypes.CDLL:
    global _LIB
    with _LOCK:
        if _LIB is None:
            path = ORACLE_DIR / "liboracle.so"
            if not path.exists():
                from . import build_oracle
                build_oracle.build_oracle()
            L = ctypes.CDLL(str(path))
            L.oracle_reduce_sum.restype = ctypes.c_double
            L.oracle_reduce_sum.argtypes = [_F, ctypes.c_size_t]
            L.oracle_softmax.argtypes = [_F, _F, ctypes.c_int, ctypes.c_int]
            L.oracle_transpose.argtypes = [_F, _F, ctypes.c_int, ctypes.c_int]
            L.oracle_rmsnorm.argtypes = [_F, _F, _F, ctypes.c_int, ctypes.c_int,
                                         ctypes.c_float]
            L.oracle_attention.argtypes = [_F, _F, _F, _F, ctypes.c_int,
                                           ctypes.c_int, ctypes.c_int,
                                           ctypes.c_int, _D]
            L.oracle_attention_rows.argtypes = [_F, _F, _F, _F, ctypes.c_int,
                                                ctypes.c_int, ctypes.c_int,
                                                ctypes.POINTER(ctypes.c_int),
                                                ctypes.c_int, _D]
            L.oracle_gemm_rows.argtypes = [_F, _F, _D] + [ctypes.c_int] * 5
            L.oracle_half_to_float.restype = ctypes.c_float
            L.oracle_half_to_float.argtypes = [ctypes.c_uint16]
            _LIB = L
    return _LIB


def ref_cpu() -> ctypes.CDLL | None:
    """The reference's own CPU loops (None when oracle/_ref was not built)."""
    global _REF_CPU
    with _LOCK:
        if _REF_CPU is None:
            path = ORACLE_DIR / "_ref" / "libref_cpu.so"
            if not path.exists():
                return None
            L = ctypes.CDLL(str(path))
            L.ref_cpu_reduce_sum.restype = ctypes.c_float
            L.ref_cpu_reduce_sum.argtypes = [_F, ctypes.c_size_t]
            L.ref_cpu_softmax.argtypes = [_F, _F, ctypes.c_int, ctypes.c_int]
            L.ref_cpu_transpose.argtypes = [_F, _F, ctypes.c_int, ctypes.c_int]
            L.ref_cpu_rmsnorm.argtypes = [_F, _F, _F, ctypes.c_int, ctypes.c_int,
                                          ctypes.c_float]
            L.ref_cpu_attention.argtypes = [_F, _F, _F, _F] + [ctypes.c_int] * 5
            _REF_CPU = L
    return _REF_CPU


def ref_gpu() -> ctypes.CDLL | None:
    """The reference's own launchers built for sm_100a (None when absent)."""
    global _REF_GPU
    with _LOCK:
        if _REF_GPU is None:
            path = ORACLE_DIR / "_ref" / "libref_operatorlib.so"
            if not path.exists():
                return None
            L = ctypes.CDLL(str(path))
            vp, i, sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t
            L.ref_reduce_sum_f32.argtypes = [vp, vp, sz, vp]
            L.ref_softmax_f32.argtypes = [vp, vp, i, i, vp]
            L.ref_transpose_f32.argtypes = [vp, vp, i, i, vp]
            L.ref_rmsnorm_f32.argtypes = [vp, vp, vp, i, i, ctypes.c_float, vp]
            L.ref_gemm_f32.argtypes = [vp, vp, vp, i, i, i, vp]
            L.ref_gemm_f16.argtypes = [vp, vp, vp, i, i, i, vp]
            L.ref_attention_f32.argtypes = [vp, vp, vp, vp, i, i, i, i, i, vp]
            L.ref_attention_f16.argtypes = [vp, vp, vp, vp, i, i, i, i, i, vp]
            _REF_GPU = L
    return _REF_GPU


def _f32(x) -> np.ndarray:
    return np.ascontiguousarray(x, dtype=np.float32)


# ---------------------------------------------------------------- oracle port

def reduce_sum(x: np.ndarray) -> float:
    x = _f32(x).ravel()
    return lib().oracle_reduce_sum(_fp(x), x.size)


def softmax(x: np.ndarray) -> np.ndarray:
    x = _f32(x)
    cols = x.shape[-1]
    rows = x.size // cols
    out = np.empty_like(x)
    lib().oracle_softmax(_fp(x), _fp(out), rows, cols)
    return out


def transpose(x: np.ndarray) -> np.ndarray:
    x = _f32(x)
    rows, cols = x.shape
    out = np.empty((cols, rows), dtype=np.float32)
    lib().oracle_transpose(_fp(x), _fp(out), rows, cols)
    return out


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = _f32(x)
    w = _f32(w)
    hidden = x.shape[-1]
    out = np.empty_like(x)
    lib().oracle_rmsnorm(_fp(x), _fp(w), _fp(out), x.size // hidden, hidden, eps)
    return out


def attention(q, k, v, causal: bool) -> np.ndarray:
    """q, k, v float32 [B,H,S,D] (FP16 callers pass the half values upcast)."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    b, h, s, d = q.shape
    out = np.empty_like(q)
    scratch = np.empty(s, dtype=np.float64)
    lib().oracle_attention(_fp(q), _fp(k), _fp(v), _fp(out), b * h, s, d,
                           int(causal), _dp(scratch))
    return out


def attention_rows(q, k, v, causal: bool, rows) -> np.ndarray:
    """Output rows `rows` of one head: q, k, v float32 [S, D]; returns
    [len(rows), D], each row computed exactly as attention() computes it."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    s, d = q.shape
    idx = np.ascontiguousarray(rows, dtype=np.int32)
    out = np.empty((idx.size, d), dtype=np.float32)
    scratch = np.empty(s, dtype=np.float64)
    lib().oracle_attention_rows(_fp(q), _fp(k), _fp(v), _fp(out), s, d, int(causal),
                                idx.ctypes.data_as(ctypes.POINTER(ctypes.c_int)),
                                idx.size, _dp(scratch))
    return out


def gemm(a: np.ndarray, b: np.ndarray, rows=None, threads: int = 1) -> np.ndarray:
    """Exact double product of float32 (or FP16-upcast) A and B; `rows`
    restricts to a row range (begin, end); `threads` splits rows."""
    a, b = _f32(a), _f32(b)
    m, k = a.shape
    n = b.shape[1]
    r0, r1 = rows if rows is not None else (0, m)
    out = np.empty((r1 - r0, n), dtype=np.float64)

    def part(lo: int, hi: int) -> None:
        view = out[lo - r0:hi - r0]
        lib().oracle_gemm_rows(_fp(a), _fp(b), _dp(view), m, n, k, lo, hi)

    if threads <= 1:
        part(r0, r1)
    else:
        bounds = np.linspace(r0, r1, threads + 1).astype(int)
        with ThreadPoolExecutor(threads) as pool:
            list(pool.map(lambda i: part(bounds[i], bounds[i + 1]), range(threads)))
    return out


def half_to_float(bits: int) -> float:
    return lib().oracle_half_to_float(bits)


def cpu_threads() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
