"""torch.ops.operatorlib.* on the GPU: the reference's own PyTorch alignment
cases and error paths (python/test_extension.py:30-168), on a non-default
stream, against the same torch oracles and tolerances it uses."""
from __future__ import annotations

import math

import pytest

pytestmark = pytest.mark.gpu


def attention_reference(q, k, v, causal):
    import torch

    scores = torch.matmul(q.float(), k.float().transpose(-1, -2)) / math.sqrt(q.size(-1))
    if causal:
        mask = torch.ones(q.size(-2), q.size(-2), device=q.device, dtype=torch.bool).triu(1)
        scores.masked_fill_(mask, -torch.inf)
    return torch.matmul(torch.softmax(scores, dim=-1), v.float())


def test_reduce_softmax(ops, stream):
    import torch

    torch.manual_seed(0)
    x = torch.randn(1_000_003, device="cuda")
    out = ops.reduce_sum(x)
    ref = x.double().sum().float()
    stream.synchronize()
    assert out.dim() == 0 and out.dtype == torch.float32
    torch.testing.assert_close(out, ref, rtol=5e-4, atol=5e-4)
    for rows, cols, scale in [(19, 128, 5.0), (17, 1024, 5.0), (17, 1003, 1000.0)]:
        x = scale * torch.randn(rows, cols, device="cuda")
        out = ops.softmax(x)
        ref = torch.softmax(x, dim=-1)
        stream.synchronize()
        torch.testing.assert_close(out, ref, rtol=1e-4, atol=1e-5)
        torch.testing.assert_close(out.sum(-1), torch.ones(rows, device="cuda"),
                                   rtol=1e-5, atol=1e-5)


def test_softmax_nd_last_dim(ops, stream):
    import torch

    x = torch.randn(2, 3, 5, 77, device="cuda")
    out = ops.softmax(x)
    stream.synchronize()
    assert out.shape == x.shape
    torch.testing.assert_close(out, torch.softmax(x, -1), rtol=1e-5, atol=1e-7)


def test_transpose_rmsnorm(ops, stream):
    import torch

    for rows, cols in [(64, 96), (65, 37)]:
        x = torch.randn(rows, cols, device="cuda")
        out = ops.transpose(x)
        stream.synchronize()
        assert torch.equal(out, x.t().contiguous())
    for shape in [(3, 7, 1024), (5, 1003)]:
        x = torch.randn(*shape, device="cuda")
        w = torch.randn(shape[-1], device="cuda")
        out = ops.rmsnorm(x, w, 1e-5)
        ref = x * torch.rsqrt(x.square().mean(-1, keepdim=True) + 1e-5) * w
        stream.synchronize()
        torch.testing.assert_close(out, ref, rtol=2e-4, atol=2e-5)
    x = torch.randn(4, 256, device="cuda")
    w = torch.randn(256, device="cuda")
    torch.testing.assert_close(ops.rmsnorm(x, w), ops.rmsnorm(x, w, 1e-5))


def test_gemm(ops, stream):
    import torch

    for dtype, m, n, k in [(torch.float32, 128, 64, 32), (torch.float32, 7, 37, 23),
                           (torch.float16, 128, 128, 32), (torch.float16, 16, 128, 32),
                           (torch.float16, 32, 32, 32), (torch.float16, 17, 19, 23),
                           (torch.float16, 256, 512, 256)]:
        a = 0.1 * torch.randn(m, k, device="cuda", dtype=dtype)
        b = 0.1 * torch.randn(k, n, device="cuda", dtype=dtype)
        out = ops.gemm(a, b)
        ref = torch.matmul(a.float(), b.float())
        stream.synchronize()
        assert out.dtype == torch.float32
        tol = 2e-2 if dtype == torch.float16 else 5e-4
        torch.testing.assert_close(out, ref, rtol=tol, atol=tol)


def test_attention(ops, stream):
    import torch

    for dtype, s, d, causal in [(torch.float32, 32, 64, False), (torch.float32, 32, 128, True),
                                (torch.float32, 37, 71, True), (torch.float16, 32, 64, False),
                                (torch.float16, 32, 128, True), (torch.float16, 37, 71, True),
                                (torch.float16, 256, 128, True), (torch.float16, 256, 64, False)]:
        shape = (1, 2, s, d)
        q = 0.25 * torch.randn(*shape, device="cuda", dtype=dtype)
        k = 0.25 * torch.randn(*shape, device="cuda", dtype=dtype)
        v = torch.randn(*shape, device="cuda", dtype=dtype)
        out = ops.attention(q, k, v, causal)
        ref = attention_reference(q, k, v, causal)
        stream.synchronize()
        assert out.dtype == torch.float32
        tol = 2e-2 if dtype == torch.float16 else 8e-4
        torch.testing.assert_close(out, ref, rtol=tol, atol=tol)


def expect_error(fn, text):
    with pytest.raises(RuntimeError) as info:
        fn()
    assert text in str(info.value), str(info.value)


def test_validation_messages(ops):
    import torch

    expect_error(lambda: ops.reduce_sum(torch.ones(8, device="cuda", dtype=torch.float16)), "float32")
    expect_error(lambda: ops.softmax(torch.randn(8, 16, device="cuda")[:, ::2]), "contiguous")
    expect_error(lambda: ops.softmax(torch.empty(3, 0, device="cuda")), "positive int32")
    expect_error(lambda: ops.transpose(torch.randn(2, 3, 4, device="cuda")), "2D")
    expect_error(lambda: ops.rmsnorm(torch.randn(3, 8, device="cuda"),
                                     torch.randn(7, device="cuda"), 1e-5), "weight length")
    expect_error(lambda: ops.rmsnorm(torch.randn(3, 8, device="cuda"),
                                     torch.randn(8, device="cuda"), 0.0), "epsilon")
    expect_error(lambda: ops.gemm(torch.randn(4, 8, device="cuda"),
                                  torch.randn(7, 5, device="cuda")), "a.size(1)")
    expect_error(lambda: ops.gemm(torch.randn(4, 8, device="cuda"),
                                  torch.randn(8, 5, device="cuda", dtype=torch.float16)),
                 "same dtype")
    bad = (1, 1, 8, 129)
    expect_error(lambda: ops.attention(torch.randn(*bad, device="cuda"),
                                       torch.randn(*bad, device="cuda"),
                                       torch.randn(*bad, device="cuda"), False), "at most 128")
    # CPU tensors never reach the binding: only the CUDA key is registered.
    with pytest.raises(NotImplementedError):
        ops.reduce_sum(torch.ones(8))


def test_work_is_on_callers_stream(ops, cuda):
    """The op enqueues on the current stream and does not synchronise: a
    kernel queued behind a long-running one on a side stream waits for it."""
    import torch

    side = torch.cuda.Stream(cuda)
    big = torch.randn(4096, 4096, device=cuda)
    torch.cuda.synchronize()
    with torch.cuda.stream(side):
        for _ in range(20):
            big = big @ big.clamp(-1e-3, 1e-3)
        x = torch.randn(64, 1024, device=cuda)
        out = ops.softmax(x)
    side.synchronize()
    torch.testing.assert_close(out, torch.softmax(x, -1), rtol=1e-5, atol=1e-7)
