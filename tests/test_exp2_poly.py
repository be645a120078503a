"""The FMA-pipe exp2 used by the tensor-core attention softmax
(csrc/attention_tc.cu, exp2_poly): re-derives its cubic from the method the
kernel names (least squares on relative error over [-1/2, 1/2] after
round-to-nearest range reduction) and checks a float32 emulation of the
kernel's exact operation sequence stays within 1e-4 relative error of 2^x --
below the FP16 half-ulp (4.9e-4) that P is rounded to."""
from __future__ import annotations

import re
from pathlib import Path

import numpy as np

SRC = Path(__file__).resolve().parents[1] / "orin-cuda-operator-library_b200" / "csrc" / "attention_tc.cu"


def kernel_coeffs():
    body = SRC.read_text().split("exp2_poly(float x)")[1].split("}")[0]
    c = [float(v) for v in re.findall(r"\b(0\.[0-9]+)f", body)]
    # fmaf(c3, f, c2); fmaf(p, f, c1); fmaf(p, f, c0)
    return c[0], c[1], c[2], c[3]


def emulate(x):
    f32 = np.float32
    c3, c2, c1, c0 = (f32(v) for v in kernel_coeffs())
    x = np.maximum(x.astype(f32), f32(-126))
    t = (x + f32(12582912.0)).astype(f32)
    n = (t - f32(12582912.0)).astype(f32)
    f = (x - n).astype(f32)
    p = (c3 * f + c2).astype(f32)
    p = (p * f + c1).astype(f32)
    p = (p * f + c0).astype(f32)
    ni = t.view(np.int32) - np.int32(0x4B400000)
    return (p.view(np.int32) + (ni << 23)).view(np.float32)


def test_fit_reproduces_kernel_coefficients():
    f = np.cos(np.linspace(0, np.pi, 2001)) * 0.5
    y = 2.0 ** f
    a = np.vstack([f ** k for k in range(4)]).T / y[:, None]
    w = np.ones_like(f)
    for _ in range(50):
        c, *_ = np.linalg.lstsq(a * w[:, None], w, rcond=None)
        err = np.abs(a @ c - 1)
        w = np.sqrt(w * (err / err.max() + 1e-3))
    c3, c2, c1, c0 = kernel_coeffs()
    np.testing.assert_allclose(c[::-1], [c3, c2, c1, c0], rtol=1e-5, atol=1e-7)


def test_relative_error_below_fp16_resolution():
    x = np.linspace(-60, 8, 2_000_001).astype(np.float32)
    got = emulate(x).astype(np.float64)
    want = np.exp2(x.astype(np.float64))
    assert np.max(np.abs(got / want - 1)) < 1e-4


def test_masked_inputs_underflow_to_zero_in_fp16():
    x = np.array([-np.inf, -1e30, -200.0, -126.0], dtype=np.float32)
    assert np.all(emulate(x).astype(np.float16) == 0)
