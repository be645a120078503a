"""Pins the CPU oracle (oracle/opl_oracle.c) to the reference.

1. Against the committed golden fixtures (outputs of the reference's own CPU
   loops, tests/golden/make_golden.py): bit-exact for every operator.
2. Against the reference's loops compiled from its sources (oracle/_ref), on
   fresh seeded inputs including the BASELINE distributions, when built.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as orc

GOLDEN = Path(__file__).resolve().parent / "golden"


def fixtures(prefix):
    files = sorted(GOLDEN.glob(f"{prefix}_*.npz"))
    assert files, f"no golden fixtures for {prefix}"
    return files


@pytest.mark.parametrize("path", fixtures("reduce"), ids=lambda p: p.stem)
def test_reduce_matches_golden(path):
    g = np.load(path)
    assert np.float32(orc.reduce_sum(g["x"])) == g["y"]


@pytest.mark.parametrize("path", fixtures("softmax"), ids=lambda p: p.stem)
def test_softmax_matches_golden(path):
    g = np.load(path)
    assert np.array_equal(orc.softmax(g["x"]), g["y"])


@pytest.mark.parametrize("path", fixtures("transpose"), ids=lambda p: p.stem)
def test_transpose_matches_golden(path):
    g = np.load(path)
    assert np.array_equal(orc.transpose(g["x"]), g["y"])


@pytest.mark.parametrize("path", fixtures("rmsnorm"), ids=lambda p: p.stem)
def test_rmsnorm_matches_golden(path):
    g = np.load(path)
    assert np.array_equal(orc.rmsnorm(g["x"], g["w"], float(g["eps"])), g["y"])


@pytest.mark.parametrize("path", fixtures("attention"), ids=lambda p: p.stem)
def test_attention_matches_golden(path):
    g = np.load(path)
    out = orc.attention(g["q"], g["k"], g["v"], bool(g["causal"]))
    assert np.array_equal(out, g["y"])


def test_half_conversion_matches_numpy():
    bits = np.arange(0, 1 << 16, 7, dtype=np.uint16)
    expect = bits.view(np.float16).astype(np.float32)
    got = np.array([orc.half_to_float(int(b)) for b in bits], dtype=np.float32)
    finite = np.isfinite(expect)
    assert np.array_equal(got[finite], expect[finite])
    assert np.array_equal(np.isnan(got), np.isnan(expect))


def test_gemm_oracle_is_exact_double_product():
    rng = np.random.default_rng(5)
    a = rng.uniform(-1, 1, (37, 71)).astype(np.float32)
    b = rng.uniform(-1, 1, (71, 65)).astype(np.float32)
    np.testing.assert_allclose(orc.gemm(a, b), a.astype(np.float64) @ b.astype(np.float64),
                               rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(orc.gemm(a, b, rows=(5, 20), threads=3),
                               (a.astype(np.float64) @ b.astype(np.float64))[5:20],
                               rtol=1e-12, atol=1e-12)


ref = orc.ref_cpu()
needs_ref = pytest.mark.skipif(ref is None, reason="oracle/_ref not built")


@needs_ref
def test_pins_against_reference_loops_on_baseline_distributions():
    rng = np.random.default_rng(99)
    F = orc._fp
    x = rng.uniform(-1, 1, 1 << 20).astype(np.float32)
    assert np.float32(orc.reduce_sum(x)) == np.float32(ref.ref_cpu_reduce_sum(F(x), x.size))

    x = rng.normal(0, 2, (64, 1024)).astype(np.float32)
    y = np.empty_like(x)
    ref.ref_cpu_softmax(F(x), F(y), 64, 1024)
    assert np.array_equal(orc.softmax(x), y)

    x = rng.normal(0, 1, (16, 4096)).astype(np.float32)
    w = rng.normal(1, 0.1, 4096).astype(np.float32)
    y = np.empty_like(x)
    ref.ref_cpu_rmsnorm(F(x), F(w), F(y), 16, 4096, np.float32(1e-6))
    assert np.array_equal(orc.rmsnorm(x, w, 1e-6), y)

    x = rng.uniform(-1, 1, (41, 1023)).astype(np.float32)
    y = np.empty((1023, 41), dtype=np.float32)
    ref.ref_cpu_transpose(F(x), F(y), 41, 1023)
    assert np.array_equal(orc.transpose(x), y)

    shape = (1, 2, 64, 128)
    q, k, v = (rng.normal(0, 1, shape).astype(np.float16).astype(np.float32)
               for _ in range(3))
    for causal in (0, 1):
        y = np.empty_like(q)
        ref.ref_cpu_attention(F(q), F(k), F(v), F(y), 1, 2, 64, 128, causal)
        assert np.array_equal(orc.attention(q, k, v, bool(causal)), y)
