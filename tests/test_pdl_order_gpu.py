"""Kernels launched with programmatic dependent launch may start while the
previous kernel on the stream still runs; each must read what that kernel
wrote only after griddepcontrol.wait.  These tests chain such launches on one
stream with no synchronisation between them, each reading the previous one's
output (or, for the reduce, reusing the same stream-ordered workspace with a
different input), and check every result against the CPU oracle."""
from __future__ import annotations

import numpy as np
import pytest

import operatorlib
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def _dev(a, cuda):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


def test_reduce_alternating_inputs_back_to_back(cuda, stream):
    """The finalize kernel must not see the partials of the previous call
    (same workspace memory, other input)."""
    import torch

    n = 16_777_216
    xs = [np.random.default_rng(40 + i).uniform(-1, 1, n).astype(np.float32) for i in range(2)]
    ds = [_dev(x, cuda) for x in xs]
    torch.cuda.synchronize()
    outs = torch.empty(8, device=cuda)
    for k in range(8):
        operatorlib.reduce_sum_into(ds[k % 2], outs[k])
    stream.synchronize()
    for k in range(8):
        want = orc.reduce_sum(xs[k % 2])
        got = outs[k].item()
        assert abs(got - want) <= 1e-6 * abs(want) + 1e-6, (k, got, want)


def test_softmax_chain_fp32(cuda, stream):
    import torch

    x = np.random.default_rng(3).normal(0, 2, (4096, 1024)).astype(np.float32)
    a = _dev(x, cuda)
    b = torch.empty_like(a)
    c = torch.empty_like(a)
    torch.cuda.synchronize()
    operatorlib.softmax_into(a, b)
    operatorlib.softmax_into(b, c)  # reads the first launch's output
    stream.synchronize()
    want = orc.softmax(orc.softmax(x).astype(np.float32))
    np.testing.assert_allclose(c.cpu().numpy(), want, rtol=1e-5, atol=1e-9)


def test_rmsnorm_chain_ragged_fp32(cuda, stream):
    """Ragged rows (warp per row, weight staged in shared memory): the
    weight of the second launch is the first launch's first output row."""
    import torch

    x = np.random.default_rng(4).normal(0, 1, (4097, 1023)).astype(np.float32)
    w = np.random.default_rng(5).normal(1, 0.1, 1023).astype(np.float32)
    a, wd = _dev(x, cuda), _dev(w, cuda)
    b = torch.empty_like(a)
    c = torch.empty_like(a)
    torch.cuda.synchronize()
    operatorlib.rmsnorm_into(a, wd, b, 1e-6)
    operatorlib.rmsnorm_into(b, b[0], c, 1e-6)
    stream.synchronize()
    first = orc.rmsnorm(x, w, 1e-6).astype(np.float32)
    want = orc.rmsnorm(first, first[0], 1e-6)
    np.testing.assert_allclose(c.cpu().numpy(), want, rtol=1e-4, atol=1e-6)


def test_softmax_chain_bf16(cuda, stream):
    import torch

    x = np.random.default_rng(6).normal(0, 2, (4096, 1024)).astype(np.float32)
    a = _dev(x, cuda).to(torch.bfloat16)
    b = torch.empty_like(a)
    c = torch.empty_like(a)
    torch.cuda.synchronize()
    operatorlib.softmax_into(a, b)
    operatorlib.softmax_into(b, c)
    stream.synchronize()
    ref = torch.softmax(torch.softmax(a.float(), -1).to(torch.bfloat16).float(), -1)
    err = (c.float() - ref).abs().max().item()
    assert err <= 2 ** -7, err
