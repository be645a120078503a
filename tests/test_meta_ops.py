"""Meta (shape-only) kernels of torch.ops.operatorlib.*, on CPU: output
shapes and dtypes follow the CUDA ops, and argument errors carry the same
texts as the CUDA path (reference python/test_extension.py:124-168)."""
from __future__ import annotations

import pytest
import torch

import operatorlib


@pytest.fixture(scope="module")
def ops():
    operatorlib.load_operatorlib()
    return torch.ops.operatorlib


def meta(*shape, dtype=torch.float32):
    return torch.empty(*shape, device="meta", dtype=dtype)


def test_shapes_and_dtypes(ops):
    assert ops.reduce_sum(meta(100)).shape == ()
    assert ops.softmax(meta(2, 3, 77)).shape == (2, 3, 77)
    assert ops.transpose(meta(5, 9)).shape == (9, 5)
    assert ops.rmsnorm(meta(4, 64), meta(64)).shape == (4, 64)
    for dt in (torch.float32, torch.float16):
        c = ops.gemm(meta(7, 11, dtype=dt), meta(11, 3, dtype=dt))
        assert c.shape == (7, 3) and c.dtype == torch.float32
        o = ops.attention(meta(2, 4, 33, 64, dtype=dt), meta(2, 4, 33, 64, dtype=dt),
                          meta(2, 4, 33, 64, dtype=dt), True)
        assert o.shape == (2, 4, 33, 64) and o.dtype == torch.float32
    assert all(t.device.type == "meta" for t in [ops.softmax(meta(2, 2))])


@pytest.mark.parametrize("call,text", [
    (lambda o: o.reduce_sum(meta(8, dtype=torch.float16)), "float32"),
    (lambda o: o.softmax(meta(3, 0)), "positive int32"),
    (lambda o: o.transpose(meta(2, 3, 4)), "2D"),
    (lambda o: o.rmsnorm(meta(3, 8), meta(7), 1e-5), "weight length"),
    (lambda o: o.rmsnorm(meta(3, 8), meta(8), -1.0), "epsilon"),
    (lambda o: o.gemm(meta(4, 8), meta(7, 5)), "a.size(1)"),
    (lambda o: o.attention(meta(1, 1, 8, 129), meta(1, 1, 8, 129), meta(1, 1, 8, 129), False),
     "at most 128"),
])
def test_meta_errors_match_cuda_texts(ops, call, text):
    with pytest.raises(RuntimeError, match=text.replace("(", r"\(").replace(")", r"\)")):
        call(ops)
