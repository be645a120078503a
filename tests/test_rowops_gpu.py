"""Parity of the bandwidth-bound operators (reduce, softmax, rmsnorm,
transpose) on the GPU, called through the C-ABI, against the CPU oracle.

Gates: FP32 row ops rel <= 1e-5 (plus a tiny absolute
floor for softmax outputs near 0); reduce within 1e-6 relative of the
double-precision sum; transpose bit-exact.  Shapes cover the reference's own
test cases (tests/core_ops_smoke.cu, python/test_extension.py), the BASELINE
configs at full size, ragged 4097x1023, tiny and very long rows, and
misaligned (non-16-byte) base pointers.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

import operatorlib
from oracle import oracle as orc

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def dev(a, cuda):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


def host(t):
    return t.cpu().numpy()


def rel_close(got, want, rtol, atol):
    np.testing.assert_allclose(got, want, rtol=rtol, atol=atol)


# ----------------------------------------------------------------- reduce

@pytest.mark.parametrize("n", [1, 2, 3, 4, 5, 17, 1000, 4096, 65537, 1_000_003,
                               16_777_216, 16_777_216 + 3])
def test_reduce_sum(cuda, stream, n):
    import torch

    x = np.random.default_rng(n).uniform(-1, 1, n).astype(np.float32)
    out = torch.empty((), device=cuda)
    operatorlib.reduce_sum_into(dev(x, cuda), out)
    stream.synchronize()
    want = orc.reduce_sum(x)
    assert abs(out.item() - want) <= 1e-6 * abs(want) + 1e-6, (out.item(), want)


def test_reduce_sum_iota_reference_case(cuda, stream):
    import torch

    x = np.arange(-500, 500, dtype=np.float32)  # core_ops_smoke.cu:33-35
    out = torch.empty((), device=cuda)
    operatorlib.reduce_sum_into(dev(x, cuda), out)
    stream.synchronize()
    assert out.item() == -500.0


@pytest.mark.parametrize("offset", [1, 2, 3])
def test_reduce_sum_misaligned_base(cuda, stream, offset):
    import torch

    x = np.random.default_rng(offset).uniform(-1, 1, 100_000).astype(np.float32)
    full = dev(x, cuda)
    view = full[offset:]
    out = torch.empty((), device=cuda)
    operatorlib.reduce_sum_into(view, out)
    stream.synchronize()
    want = orc.reduce_sum(x[offset:])
    assert abs(out.item() - want) <= 1e-6 * abs(want) + 1e-6


def test_reduce_sum_deterministic(cuda, stream):
    import torch

    x = dev(np.random.default_rng(3).normal(0, 1, 5_000_000).astype(np.float32), cuda)
    outs = []
    for _ in range(5):
        o = torch.empty((), device=cuda)
        operatorlib.reduce_sum_into(x, o)
        outs.append(o)
    stream.synchronize()
    assert len({o.item() for o in outs}) == 1


def test_reduce_partial_f64(cuda, stream):
    import torch

    x = np.random.default_rng(8).uniform(-1, 1, 3_000_001).astype(np.float32)
    out = torch.empty((), device=cuda, dtype=torch.float64)
    operatorlib.reduce_sum_partial_f64_into(dev(x, cuda), out)
    stream.synchronize()
    want = orc.reduce_sum(x)
    assert abs(out.item() - want) <= 1e-6 * abs(want) + 1e-6


@pytest.mark.parametrize("path", sorted(GOLDEN.glob("reduce_*.npz")), ids=lambda p: p.stem)
def test_reduce_golden(cuda, stream, path):
    import torch

    g = np.load(path)
    out = torch.empty((), device=cuda)
    operatorlib.reduce_sum_into(dev(g["x"], cuda), out)
    stream.synchronize()
    assert abs(out.item() - float(g["y"])) <= 1e-6 * abs(float(g["y"])) + 1e-6


# ----------------------------------------------------------------- softmax

SOFTMAX_CASES = [
    (19, 128, 5.0), (17, 1024, 5.0), (17, 1003, 1000.0),  # reference tests
    (4096, 1024, 2.0),                                    # BASELINE config
    (4097, 1023, 2.0),                                    # ragged config
    (1, 1, 1.0), (3, 7, 1.0), (33, 33, 3.0), (8, 2048, 2.0), (5, 4100, 2.0),
    (3, 8192, 2.0), (2, 16383, 2.0), (2, 32768, 2.0), (2, 40000, 2.0),
    (1, 100_003, 2.0),
    (5, 5, 2.0), (11, 130, 2.0), (6, 2047, 2.0), (9, 2163, 2.0),  # ragged float4 windows
]


@pytest.mark.parametrize("rows,cols,scale", SOFTMAX_CASES)
def test_softmax(cuda, stream, rows, cols, scale):
    import torch

    x = np.random.default_rng(rows * 7 + cols).normal(0, scale, (rows, cols)).astype(np.float32)
    y = torch.empty((rows, cols), device=cuda)
    operatorlib.softmax_into(dev(x, cuda), y)
    stream.synchronize()
    got = host(y)
    rel_close(got, orc.softmax(x), rtol=1e-5, atol=1e-9)
    np.testing.assert_allclose(got.astype(np.float64).sum(axis=1), 1.0, atol=2e-5)


@pytest.mark.parametrize("path", sorted(GOLDEN.glob("softmax_*.npz")), ids=lambda p: p.stem)
def test_softmax_golden(cuda, stream, path):
    import torch

    g = np.load(path)
    y = torch.empty(g["x"].shape, device=cuda)
    operatorlib.softmax_into(dev(g["x"], cuda), y)
    stream.synchronize()
    rel_close(host(y), g["y"], rtol=1e-5, atol=1e-9)


def test_softmax_misaligned_rows_use_scalar_path(cuda, stream):
    import torch

    x = np.random.default_rng(2).normal(0, 2, 64 * 512 + 1).astype(np.float32)
    t = dev(x, cuda)[1:].view(64, 512)  # 4-byte offset base
    y = torch.empty(64 * 512 + 1, device=cuda)[1:].view(64, 512)
    operatorlib.softmax_into(t, y)
    stream.synchronize()
    rel_close(host(y), orc.softmax(x[1:].reshape(64, 512)), rtol=1e-5, atol=1e-9)


# ----------------------------------------------------------------- rmsnorm

RMS_CASES = [(32, 4096), (17, 1003), (3 * 7, 1024), (5, 1003),  # reference tests
             (2048, 4096),                                       # BASELINE
             (4097, 1023),                                       # ragged
             (1, 1), (9, 3), (4, 64), (7, 8192), (3, 16384), (2, 30001),
             (2, 32768), (2, 40000), (1, 131_072),
             (4, 5), (13, 513), (6, 2047), (9, 2163)]  # ragged float4 windows


@pytest.mark.parametrize("tokens,hidden", RMS_CASES)
def test_rmsnorm(cuda, stream, tokens, hidden):
    import torch

    rng = np.random.default_rng(tokens + hidden)
    x = rng.normal(0, 1, (tokens, hidden)).astype(np.float32)
    w = rng.normal(1, 0.1, hidden).astype(np.float32)
    y = torch.empty((tokens, hidden), device=cuda)
    operatorlib.rmsnorm_into(dev(x, cuda), dev(w, cuda), y, 1e-6)
    stream.synchronize()
    rel_close(host(y), orc.rmsnorm(x, w, 1e-6), rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("path", sorted(GOLDEN.glob("rmsnorm_*.npz")), ids=lambda p: p.stem)
def test_rmsnorm_golden(cuda, stream, path):
    import torch

    g = np.load(path)
    y = torch.empty(g["x"].shape, device=cuda)
    operatorlib.rmsnorm_into(dev(g["x"], cuda), dev(g["w"], cuda), y, float(g["eps"]))
    stream.synchronize()
    rel_close(host(y), g["y"], rtol=1e-5, atol=1e-7)


# ----------------------------------------------------------------- transpose

T_CASES = [(37, 65), (64, 96), (65, 37), (4096, 4096), (4097, 1023), (1, 1),
           (1, 1000), (1000, 1), (4, 4), (8, 12), (64, 64), (68, 132),
           (3, 100_000), (100_000, 3), (1024, 4100),
           # taller than 65535 row tiles: the grid loops over row tiles
           (5_000_000, 4), (5_000_001, 3)]


@pytest.mark.parametrize("rows,cols", T_CASES)
def test_transpose_bit_exact(cuda, stream, rows, cols):
    import torch

    x = np.random.default_rng(rows ^ cols).uniform(-1, 1, (rows, cols)).astype(np.float32)
    y = torch.empty((cols, rows), device=cuda)
    operatorlib.transpose_into(dev(x, cuda), y)
    stream.synchronize()
    assert np.array_equal(host(y).view(np.uint32), np.ascontiguousarray(x.T).view(np.uint32))


def test_transpose_preserves_nan_payload_bits(cuda, stream):
    import torch

    bits = np.random.default_rng(1).integers(0, 2**32, (128, 96), dtype=np.uint64).astype(np.uint32)
    x = bits.view(np.float32)
    y = torch.empty((96, 128), device=cuda)
    operatorlib.transpose_into(dev(x, cuda), y)
    stream.synchronize()
    assert np.array_equal(host(y).view(np.uint32), np.ascontiguousarray(bits.T))


@pytest.mark.parametrize("path", sorted(GOLDEN.glob("transpose_*.npz")), ids=lambda p: p.stem)
def test_transpose_golden(cuda, stream, path):
    import torch

    g = np.load(path)
    y = torch.empty(g["y"].shape, device=cuda)
    operatorlib.transpose_into(dev(g["x"], cuda), y)
    stream.synchronize()
    assert np.array_equal(host(y), g["y"])


# ------------------------------------------ same inputs through the reference

def test_against_reference_kernels_on_b200(cuda, stream):
    """The reference's own launchers, built for sm_100a from its sources
    (oracle/_ref), agree with ours within the gates on the BASELINE shapes."""
    import torch

    ref = orc.ref_gpu()
    if ref is None:
        pytest.skip("oracle/_ref not built")
    s = stream.cuda_stream
    rng = np.random.default_rng(11)
    x = dev(rng.normal(0, 2, (4096, 1024)).astype(np.float32), cuda)
    a, b = torch.empty_like(x), torch.empty_like(x)
    operatorlib.softmax_into(x, a)
    assert ref.ref_softmax_f32(x.data_ptr(), b.data_ptr(), 4096, 1024, s) == 0
    x2 = dev(rng.uniform(-1, 1, (4096, 4096)).astype(np.float32), cuda)
    c, d = torch.empty_like(x2), torch.empty_like(x2)
    operatorlib.transpose_into(x2, c)
    assert ref.ref_transpose_f32(x2.data_ptr(), d.data_ptr(), 4096, 4096, s) == 0
    stream.synchronize()
    rel_close(host(a), host(b), rtol=1e-5, atol=1e-8)
    assert torch.equal(c, d)
