"""The allocation-free reduce entry point, opl_reduce_sum_f32_noalloc.

It exists for callers that must not allocate device memory (allocator hooks,
pool callbacks, frameworks owning all device memory).  Called through the
C-ABI, it must give the same sums as opl_reduce_sum_f32 -- within the reduce
gate used everywhere in these tests (1e-6 relative) -- on two calls in a row,
the second reusing the shared scratch array the first one filled.  This file
is collected last so a stop-at-first-failure run has done everything else.
"""
from __future__ import annotations


import numpy as np
import pytest

import operatorlib

pytestmark = pytest.mark.gpu


def test_noalloc_matches_allocating_entry_point(cuda):
    import torch

    lib = operatorlib.capi()
    stream = torch.cuda.Stream(cuda)
    handle = stream.cuda_stream
    rng = np.random.default_rng(2024)
    for n in (16_777_216, 1_000_003):  # two calls in a row, different sizes
        x = torch.from_numpy(rng.uniform(-1, 1, n).astype(np.float32)).to(cuda)
        torch.cuda.synchronize()
        got = torch.empty((), device=cuda)
        want = torch.empty((), device=cuda)
        assert lib.opl_reduce_sum_f32_noalloc(x.data_ptr(), got.data_ptr(), n, handle) == 0
        assert lib.opl_reduce_sum_f32(x.data_ptr(), want.data_ptr(), n, handle) == 0
        stream.synchronize()
        w = want.item()
        assert abs(got.item() - w) <= 1e-6 * abs(w) + 1e-6, (n, got.item(), w)


def test_noalloc_rejects_bad_arguments():
    lib = operatorlib.capi()
    assert lib.opl_reduce_sum_f32_noalloc(None, 0x1000, 10, None) == 1
    assert lib.opl_reduce_sum_f32_noalloc(0x1000, 0x1000, 0, None) == 1
