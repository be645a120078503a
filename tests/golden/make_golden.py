"""Generates tests/golden/*.npz: seeded inputs and the outputs of the
REFERENCE's own CPU verification loops on them.

The loops come from oracle/_ref/libref_cpu.so, which oracle/build_oracle.py
compiles from the reference's standalone sources where they lie (reduce
reduce_v3.cu:125-128, softmax softmax_v4.cu:253-268, transpose
transpose_v2.cu:104-113, rmsnorm rmsnorm_v3.cu:154-172, attention
attention_common.h:123-156).  Case shapes follow the reference's own tests
(tests/core_ops_smoke.cu, tests/attention_smoke.cu, python/test_extension.py).
The fixtures pin the C restatement in oracle/opl_oracle.c where the reference
tree is absent.

Run: python tests/golden/make_golden.py   (needs oracle/_ref built)
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))
from oracle import oracle as orc  # noqa: E402

F = orc._fp


def main() -> int:
    ref = orc.ref_cpu()
    if ref is None:
        print("oracle/_ref/libref_cpu.so not built", file=sys.stderr)
        return 1
    rng = np.random.default_rng(20260809)
    cases = {}

    # reduce: the reference's iota case (core_ops_smoke.cu:33-35) and uniforms
    for name, x in {
        "iota1000": np.arange(-500, 500, dtype=np.float32),
        "uniform4097": rng.uniform(-1, 1, 4097).astype(np.float32),
        "uniform65536": rng.uniform(-0.5, 0.5, 65536).astype(np.float32),
    }.items():
        cases[f"reduce_{name}"] = dict(
            x=x, y=np.float32(ref.ref_cpu_reduce_sum(F(x), x.size)))

    # softmax: shapes and ranges of core_ops_smoke.cu:171-174 /
    # test_extension.py:36-37
    for rows, cols, rng_ in [(19, 128, 5.0), (17, 1024, 5.0), (17, 1003, 1000.0),
                             (5, 33, 1.0)]:
        x = rng.uniform(-rng_, rng_, (rows, cols)).astype(np.float32)
        y = np.empty_like(x)
        ref.ref_cpu_softmax(F(x), F(y), rows, cols)
        cases[f"softmax_{rows}x{cols}"] = dict(x=x, y=y)

    for rows, cols in [(37, 65), (64, 96), (65, 37)]:
        x = rng.uniform(-100, 100, (rows, cols)).astype(np.float32)
        y = np.empty((cols, rows), dtype=np.float32)
        ref.ref_cpu_transpose(F(x), F(y), rows, cols)
        cases[f"transpose_{rows}x{cols}"] = dict(x=x, y=y)

    # rmsnorm: core_ops_smoke.cu:121-164 ranges
    for tokens, hidden in [(8, 4096), (17, 1003), (3, 1024)]:
        x = rng.uniform(-3, 3, (tokens, hidden)).astype(np.float32)
        w = rng.uniform(0.5, 1.5, hidden).astype(np.float32)
        y = np.empty_like(x)
        ref.ref_cpu_rmsnorm(F(x), F(w), F(y), tokens, hidden, np.float32(1e-5))
        cases[f"rmsnorm_{tokens}x{hidden}"] = dict(x=x, w=w, y=y, eps=np.float32(1e-5))

    # attention: attention_smoke.cu cases (S32 D64, S32 D128 causal, S37 D71
    # causal with q/k in +-20), two heads
    for s, d, causal, qk in [(32, 64, 0, 1.0), (32, 128, 1, 1.0), (37, 71, 1, 20.0)]:
        shape = (1, 2, s, d)
        q = rng.uniform(-qk, qk, shape).astype(np.float32)
        k = rng.uniform(-qk, qk, shape).astype(np.float32)
        v = rng.uniform(-1, 1, shape).astype(np.float32)
        y = np.empty_like(q)
        ref.ref_cpu_attention(F(q), F(k), F(v), F(y), 1, 2, s, d, causal)
        cases[f"attention_s{s}d{d}c{causal}"] = dict(q=q, k=k, v=v, y=y,
                                                     causal=np.int32(causal))

    for name, arrays in cases.items():
        np.savez_compressed(HERE / f"{name}.npz", **arrays)
    print(f"wrote {len(cases)} fixtures to {HERE}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
