"""Tensor-level calls straight onto the C-ABI (no torch binding involved).

Each ``*_into`` function takes contiguous CUDA tensors with preallocated
outputs, passes their device pointers and the current CUDA stream (or
``stream``) to the matching ``opl_*`` entry point and raises ``OplError`` on a
non-zero return -- the same contract a C, cgo or JNI caller gets.
"""
from __future__ import annotations


def _ptr(t) -> int:
    return t.data_ptr()


def _stream(t, stream) -> int:
    import torch

    s = stream if stream is not None else torch.cuda.current_stream(t.device)
    return s.cuda_stream


def _lib():
    from . import capi

    return capi()


def _check(op, code):
    from . import check

    check(op, code)


def reduce_sum_into(x, out, stream=None) -> None:
    _check("reduce_sum", _lib().opl_reduce_sum_f32(
        _ptr(x), _ptr(out), x.numel(), _stream(x, stream)))


def reduce_sum_partial_f64_into(x, out, stream=None) -> None:
    _check("reduce_sum_partial_f64", _lib().opl_reduce_sum_partial_f64(
        _ptr(x), _ptr(out), x.numel(), _stream(x, stream)))


def _dtype_fn(base: str, dtype):
    import torch

    suffix = {torch.float32: "f32", torch.float16: "f16", torch.bfloat16: "bf16"}[dtype]
    return getattr(_lib(), f"opl_{base}_{suffix}")


def softmax_into(x, out, stream=None) -> None:
    """FP32, FP16 or BF16 (out has x's dtype; arithmetic in FP32)."""
    cols = x.shape[-1]
    _check("softmax", _dtype_fn("softmax", x.dtype)(
        _ptr(x), _ptr(out), x.numel() // cols, cols, _stream(x, stream)))


def transpose_into(x, out, stream=None) -> None:
    rows, cols = x.shape
    _check("transpose", _lib().opl_transpose_f32(
        _ptr(x), _ptr(out), rows, cols, _stream(x, stream)))


def rmsnorm_into(x, w, out, eps: float, stream=None) -> None:
    """FP32, FP16 or BF16 (w and out have x's dtype; arithmetic in FP32)."""
    hidden = x.shape[-1]
    _check("rmsnorm", _dtype_fn("rmsnorm", x.dtype)(
        _ptr(x), _ptr(w), _ptr(out), x.numel() // hidden, hidden, float(eps),
        _stream(x, stream)))


def gemm_into(a, b, c, stream=None) -> None:
    import torch

    m, k = a.shape
    n = b.shape[1]
    fn = _lib().opl_gemm_f16 if a.dtype == torch.float16 else _lib().opl_gemm_f32
    _check("gemm", fn(_ptr(a), _ptr(b), _ptr(c), m, n, k, _stream(a, stream)))


def attention_into(q, k, v, out, causal: bool, stream=None) -> None:
    import torch

    b, h, s, d = q.shape
    fn = (_lib().opl_attention_f16 if q.dtype == torch.float16
          else _lib().opl_attention_f32)
    _check("attention", fn(_ptr(q), _ptr(k), _ptr(v), _ptr(out), b, h, s, d,
                           int(bool(causal)), _stream(q, stream)))
