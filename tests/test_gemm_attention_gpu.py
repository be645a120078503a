"""Parity of GEMM and attention on the GPU through the C-ABI.

Oracles: the exact double GEMM product and the reference's double attention
loop restated in oracle/opl_oracle.c (pinned in test_oracle_pins.py).
Gates: FP16 GEMM / attention max-abs <= 2e-2 and rel <= 1e-2 against the
FP64 reference; FP32 GEMM 1e-3 + 1e-3*|ref| (reference
tests/gemm_smoke.cu:76); FP32 attention atol = rtol = 1e-4 (reference
tests/attention_smoke.cu:108).  FP16 inputs are quantised to half before the
oracle sees them, as the reference does (attention_fp16_common.h:15-22).
"""
from __future__ import annotations

import numpy as np
import pytest

import operatorlib
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def dev(a, cuda):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


def run_gemm(cuda, stream, a, b):
    import torch

    c = torch.empty((a.shape[0], b.shape[1]), device=cuda)
    operatorlib.gemm_into(dev(a, cuda), dev(b, cuda), c)
    stream.synchronize()
    return c.cpu().numpy()


def check_f16(got, want):
    err = np.abs(got.astype(np.float64) - want)
    assert err.max() <= 2e-2, err.max()
    assert np.all(err <= 2e-2 * np.abs(want) + 2e-2)
    fro = np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-30)
    assert fro <= 1e-2, fro


GEMM_F16 = [(128, 128, 32), (16, 128, 32), (32, 32, 32), (37, 65, 71),  # ref tests
            (17, 19, 23), (1, 256, 64), (1, 1, 1), (128, 256, 64), (256, 512, 1024),
            (1000, 1000, 1000), (512, 4096, 4096), (4095, 4097, 4093),
            (4096, 4096, 4096), (300, 520, 136), (129, 257, 72),
            # narrow N remainders: 256-wide kernel + skinny-N tail product
            (1000, 4104, 512), (257, 300, 64), (200, 320, 96), (129, 513, 1000),
            (640, 769, 333),
            # ragged K with a remainder of <= 8 columns: computed in A's padding pass
            (300, 262, 77), (200, 520, 45), (1000, 1033, 999),
            # larger padded products (both operands / a 1-column remainder)
            (2048, 2304, 2050), (2304, 2561, 1999),
            # padded rows too long for the bulk-copy ring: per-row fallback
            (256, 264, 26001), (300, 26001, 64)]


@pytest.mark.parametrize("m,n,k", GEMM_F16)
def test_gemm_f16(cuda, stream, m, n, k):
    rng = np.random.default_rng(m * 31 + n * 7 + k)
    a = (rng.uniform(-1, 1, (m, k)) / np.sqrt(k)).astype(np.float16)
    b = (rng.uniform(-1, 1, (k, n)) / np.sqrt(k)).astype(np.float16)
    got = run_gemm(cuda, stream, a, b)
    if m * n * k <= 2**31:
        want = orc.gemm(a.astype(np.float32), b.astype(np.float32), threads=8)
        check_f16(got, want)
    else:  # sample 96 rows spread over M for the big shapes
        idx = np.unique(np.linspace(0, m - 1, 96).astype(int))
        want = a[idx].astype(np.float64) @ b.astype(np.float64)
        check_f16(got[idx], want)


GEMM_F32 = [(1, 256, 64), (16, 128, 64), (128, 64, 32), (37, 65, 71),  # ref tests
            (7, 37, 23), (128, 128, 8), (1, 1, 1), (513, 257, 129),
            (1024, 1024, 1024), (4095, 4097, 4093),
            # > 2 tiles per SM with a small last wave: K-split tail tiles
            (2048, 2560, 256), (2048, 2600, 200)]


def test_gemm_f32_split_tail_deterministic(cuda, stream):
    """Tail tiles computed as two K halves added into a zeroed C: repeat
    runs are bit-identical."""
    import torch

    rng = np.random.default_rng(5)
    m, n, k = 2048, 2560, 512
    a = torch.from_numpy((rng.uniform(-1, 1, (m, k)) / np.sqrt(k)).astype(np.float32)).to(cuda)
    b = torch.from_numpy((rng.uniform(-1, 1, (k, n)) / np.sqrt(k)).astype(np.float32)).to(cuda)
    outs = []
    for _ in range(3):
        c = torch.full((m, n), float("nan"), device=cuda)
        operatorlib.gemm_into(a, b, c)
        outs.append(c)
    stream.synchronize()
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])
    idx = np.unique(np.linspace(0, m - 1, 64).astype(int))
    want = a.cpu().numpy()[idx].astype(np.float64) @ b.cpu().numpy().astype(np.float64)
    np.testing.assert_allclose(outs[0].cpu().numpy()[idx], want, rtol=1e-3, atol=1e-3)


@pytest.mark.parametrize("m,n,k", GEMM_F32)
def test_gemm_f32(cuda, stream, m, n, k):
    rng = np.random.default_rng(m + n + k)
    a = rng.uniform(-0.25, 0.25, (m, k)).astype(np.float32)
    b = rng.uniform(-0.25, 0.25, (k, n)).astype(np.float32)
    got = run_gemm(cuda, stream, a, b)
    if m * n * k <= 2**31:
        want = orc.gemm(a, b, threads=8)
        np.testing.assert_allclose(got, want, rtol=1e-3, atol=1e-3)
    else:
        idx = np.unique(np.linspace(0, m - 1, 64).astype(int))
        want = a[idx].astype(np.float64) @ b.astype(np.float64)
        np.testing.assert_allclose(got[idx], want, rtol=1e-3, atol=1e-3)


def run_attention(cuda, stream, q, k, v, causal):
    import torch

    o = torch.empty(q.shape, device=cuda)
    operatorlib.attention_into(dev(q, cuda), dev(k, cuda), dev(v, cuda), o, causal)
    stream.synchronize()
    return o.cpu().numpy()


ATT_CASES = [  # (B, H, S, D, causal, qk range)
    (1, 2, 32, 64, False, 1.0), (1, 2, 32, 128, True, 1.0),  # reference tests
    (1, 2, 37, 71, True, 20.0),                              # "extreme"
    (1, 1, 1, 1, False, 1.0), (2, 3, 17, 16, True, 1.0), (1, 2, 128, 128, False, 1.0),
    (1, 2, 200, 128, True, 1.0), (1, 4, 256, 64, True, 1.0), (2, 2, 513, 96, False, 1.0),
    (1, 12, 1024, 128, False, None), (1, 12, 1024, 128, True, None),  # BASELINE
    (1, 1, 2048, 128, True, None), (1, 2, 1536, 64, False, None),   # many KV splits
    (1, 1, 1000, 128, True, None), (1, 3, 640, 64, True, None),  # causal key-range parts
    (1, 4, 300, 32, True, None), (1, 2, 700, 80, False, None),     # head_dim padded to
    (2, 2, 129, 120, True, None),                                  # 64 / 128 by TMA
]


def att_inputs(shape, qk, seed, dtype):
    rng = np.random.default_rng(seed)
    if qk is None:  # BASELINE: Q/K/V ~ N(0,1)
        q, k, v = (rng.normal(0, 1, shape) for _ in range(3))
    else:
        q = rng.uniform(-qk, qk, shape)
        k = rng.uniform(-qk, qk, shape)
        v = rng.uniform(-1, 1, shape)
    return [x.astype(dtype) for x in (q, k, v)]


@pytest.mark.parametrize("h,s,d", [(100, 520, 64), (80, 1000, 128)])
def test_attention_f16_pairs_causal(cuda, stream, h, s, d):
    """Grids with B*H*(query tiles / 2) >= 2 x SMs run two query tiles per
    CTA (the sharded-config path); causal with a ragged last tile.  A few
    heads spread over the batch are checked against the oracle."""
    q, k, v = att_inputs((1, h, s, d), None, h + s + d, np.float16)
    got = run_attention(cuda, stream, q, k, v, True)
    heads = [0, h // 3, h // 2 + 1, h - 1]
    want = orc.attention(q[:, heads].astype(np.float32), k[:, heads].astype(np.float32),
                         v[:, heads].astype(np.float32), True)
    check_f16(got[:, heads], want)


@pytest.mark.parametrize("b,h,s,d,causal,qk", ATT_CASES)
def test_attention_f16(cuda, stream, b, h, s, d, causal, qk):
    q, k, v = att_inputs((b, h, s, d), qk, s * 3 + d, np.float16)
    got = run_attention(cuda, stream, q, k, v, causal)
    want = orc.attention(q.astype(np.float32), k.astype(np.float32),
                         v.astype(np.float32), causal)
    check_f16(got, want)


@pytest.mark.parametrize("b,h,s,d,causal,qk", ATT_CASES[:9])
def test_attention_f32(cuda, stream, b, h, s, d, causal, qk):
    q, k, v = att_inputs((b, h, s, d), qk, s * 5 + d, np.float32)
    got = run_attention(cuda, stream, q, k, v, causal)
    want = orc.attention(q, k, v, causal)
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("b,h,s,d,causal,qk", ATT_CASES[11:] + [
    (1, 1, 4096, 64, False, None), (1, 1, 3001, 128, True, None)])
def test_attention_f32_balanced_ranges(cuda, stream, b, h, s, d, causal, qk):
    """Grids of fewer (head, query block) units than SMs run the balanced
    schedule: every CTA takes an equal range of all KV tiles, so one unit can
    be shared by up to 8 CTAs whose parts are merged afterwards (long rows,
    few heads, ragged S, padded head_dim)."""
    q, k, v = att_inputs((b, h, s, d), qk, s * 3 + d, np.float32)
    got = run_attention(cuda, stream, q, k, v, causal)
    want = orc.attention(q, k, v, causal)
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-4)


def test_attention_f32_baseline_shape_all_heads(cuda, stream):
    """BASELINE FP32 attention B1 H12 S1024 D128: every head, both masks,
    against the oracle's full loop (reference gate atol = rtol = 1e-4)."""
    q, k, v = att_inputs((1, 12, 1024, 128), None, 77, np.float32)
    for causal in (False, True):
        got = run_attention(cuda, stream, q, k, v, causal)
        want = orc.attention(q, k, v, causal)
        np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-4)


def test_gemm_f32_baseline_4096(cuda, stream):
    """BASELINE FP32 GEMM at exactly 4096^3 (FFMA), 64 rows spread over M
    against the FP64 product, reference gate 1e-3 + 1e-3 |ref|."""
    rng = np.random.default_rng(4096)
    a = (rng.uniform(-1, 1, (4096, 4096)) / 64).astype(np.float32)
    b = (rng.uniform(-1, 1, (4096, 4096)) / 64).astype(np.float32)
    got = run_gemm(cuda, stream, a, b)
    idx = np.unique(np.linspace(0, 4095, 64).astype(int))
    want = a[idx].astype(np.float64) @ b.astype(np.float64)
    np.testing.assert_allclose(got[idx], want, rtol=1e-3, atol=1e-3)


def test_attention_f16_sharded_config_sampled(cuda, stream):
    """Sharded config B8 H32 S4096 D128 causal FP16 at full size: 8 heads
    spread over B*H, 48 query rows each (first, last and spread rows, so
    every causal key range length is represented), against the oracle's
    per-row loop on the half-quantised inputs."""
    import torch

    b, h, s, d = 8, 32, 4096, 128
    gen = torch.Generator(device=cuda)
    gen.manual_seed(8324)
    q, k, v = (torch.randn((b, h, s, d), device=cuda, generator=gen).half() for _ in range(3))
    o = torch.empty((b, h, s, d), device=cuda)
    operatorlib.attention_into(q, k, v, o, True)
    stream.synchronize()
    rows = np.unique(np.r_[0, 1, 127, 128, s - 1, np.linspace(2, s - 2, 43).astype(int)])
    for flat in np.unique(np.linspace(0, b * h - 1, 8).astype(int)):
        bi, hi = divmod(int(flat), h)
        qh, kh, vh = (x[bi, hi].float().cpu().numpy() for x in (q, k, v))
        want = orc.attention_rows(qh, kh, vh, True, rows)
        got = o[bi, hi][torch.from_numpy(rows).to(cuda)].cpu().numpy()
        check_f16(got, want.astype(np.float64))


def test_gemm_f16_sharded_config_sampled(cuda, stream):
    """Sharded config GEMM FP16 16384^3 at full size (1 GiB of C): 32 rows
    spread over M against the FP64 product."""
    import torch

    m = n = k = 16384
    gen = torch.Generator(device=cuda)
    gen.manual_seed(16384)
    a = ((torch.rand((m, k), device=cuda, generator=gen) * 2 - 1) / 128).half()
    bm = ((torch.rand((k, n), device=cuda, generator=gen) * 2 - 1) / 128).half()
    c = torch.empty((m, n), device=cuda)
    operatorlib.gemm_into(a, bm, c)
    stream.synchronize()
    idx = torch.from_numpy(np.unique(np.linspace(0, m - 1, 32).astype(int))).to(cuda)
    want = a[idx].cpu().numpy().astype(np.float64) @ bm.cpu().numpy().astype(np.float64)
    check_f16(c[idx].cpu().numpy(), want)
    del a, bm, c
    torch.cuda.empty_cache()


@pytest.mark.parametrize("b,h,s,d,causal", [
    (4, 40, 640, 128, True),    # 160 heads x 3 tile pairs, last pair single
    (8, 20, 512, 64, False),    # D = 64
    (2, 80, 768, 128, False),
])
def test_attention_f16_paired_tiles_sampled_heads(cuda, stream, b, h, s, d, causal):
    """Grids big enough for the two-query-tiles-per-CTA schedule; the oracle
    checks a spread of heads."""
    q, k, v = att_inputs((b, h, s, d), None, b * h + s + d, np.float16)
    got = run_attention(cuda, stream, q, k, v, causal).reshape(b * h, s, d)
    idx = np.unique(np.linspace(0, b * h - 1, 5).astype(int))
    qf, kf, vf = (x.reshape(b * h, s, d)[idx][None].astype(np.float32) for x in (q, k, v))
    want = orc.attention(qf, kf, vf, causal)[0]
    check_f16(got[idx], want)


@pytest.mark.parametrize("m,n,k,offset,b_offset", [
    (64, 72, 40, 1, 1), (300, 200, 136, 3, 3), (129, 257, 72, 5, 5), (1000, 1000, 1000, 7, 7),
    # only A misaligned, N a multiple of 256 plus <= 8: B stays in place and
    # the remainder columns are computed in A's padding pass
    (300, 264, 64, 3, 0), (129, 520, 136, 1, 0),
    # larger products with only A padded / only B padded
    (2048, 2048, 2048, 3, 0), (2048, 2048, 2048, 0, 5)])
def test_gemm_f16_misaligned_base_pointers(cuda, stream, m, n, k, offset, b_offset):
    """A starts `offset` halves and B `b_offset` halves into their allocations
    (2-byte aligned only): the zero-padded staging path must read them
    correctly."""
    import torch

    rng = np.random.default_rng(m + offset)
    a = (rng.uniform(-1, 1, (m, k)) / np.sqrt(k)).astype(np.float16)
    b = (rng.uniform(-1, 1, (k, n)) / np.sqrt(k)).astype(np.float16)
    a_full = torch.zeros(m * k + offset, dtype=torch.float16, device=cuda)
    b_full = torch.zeros(k * n + b_offset, dtype=torch.float16, device=cuda)
    a_full[offset:] = torch.from_numpy(a.ravel()).to(cuda)
    b_full[b_offset:] = torch.from_numpy(b.ravel()).to(cuda)
    c = torch.empty((m, n), device=cuda)
    operatorlib.gemm_into(a_full[offset:].view(m, k), b_full[b_offset:].view(k, n), c)
    stream.synchronize()
    check_f16(c.cpu().numpy(), orc.gemm(a.astype(np.float32), b.astype(np.float32), threads=8))


@pytest.mark.parametrize("m,n,k", [(4096, 4096, 4096), (4095, 4097, 4093), (2048, 2304, 1024), (1280, 2560, 1024),
                                   (2304, 2561, 1999)])
def test_gemm_f16_deterministic(cuda, stream, m, n, k):
    """Shapes whose last wave is split into K halves (added into a zeroed C)
    still give bit-identical results run to run."""
    import torch

    rng = np.random.default_rng(9)
    a = torch.from_numpy((rng.uniform(-1, 1, (m, k)) / np.sqrt(k)).astype(np.float16)).to(cuda)
    b = torch.from_numpy((rng.uniform(-1, 1, (k, n)) / np.sqrt(k)).astype(np.float16)).to(cuda)
    outs = []
    for _ in range(3):
        c = torch.empty((m, n), device=cuda)
        operatorlib.gemm_into(a, b, c)
        outs.append(c)
    stream.synchronize()
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])
    idx = np.unique(np.linspace(0, m - 1, 40).astype(int))
    want = a.cpu().numpy()[idx].astype(np.float64) @ b.cpu().numpy().astype(np.float64)
    check_f16(outs[0].cpu().numpy()[idx], want)


@pytest.mark.parametrize("m,n,k", [(1, 4096, 4096), (2, 1000, 4096), (3, 4104, 333), (8, 2048, 2048),
                                   (16, 4096, 4096), (16, 8, 7), (5, 8192, 64), (1, 64, 100_000),
                                   (17, 4096, 1024), (32, 2048, 4096), (40, 1000, 520),
                                   (64, 4096, 4096), (100, 8, 64), (128, 4096, 4096),
                                   (128, 16384, 512), (1, 128, 8), (7, 136, 72)])
def test_gemm_f16_skinny(cuda, stream, m, n, k):
    """Skinny M <= 128: swapped-operand tensor-core kernel with a cluster
    split-K (K % 8 == 0), split-K SIMT kernel otherwise; FP16 gates and
    bit-identical repeat runs."""
    import torch

    rng = np.random.default_rng(m * 7 + n + k)
    a = (rng.uniform(-1, 1, (m, k)) / np.sqrt(k)).astype(np.float16)
    b = (rng.uniform(-1, 1, (k, n)) / np.sqrt(k)).astype(np.float16)
    ad, bd = dev(a, cuda), dev(b, cuda)
    c1 = torch.empty((m, n), device=cuda)
    c2 = torch.empty((m, n), device=cuda)
    operatorlib.gemm_into(ad, bd, c1)
    operatorlib.gemm_into(ad, bd, c2)
    stream.synchronize()
    assert torch.equal(c1, c2)
    check_f16(c1.cpu().numpy(), a.astype(np.float64) @ b.astype(np.float64))
