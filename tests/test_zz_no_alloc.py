"""The allocation-free reduce entry point, opl_reduce_sum_f32_noalloc.

It exists for callers that must not allocate device memory (allocator hooks,
pool callbacks, frameworks owning all device memory).  Called through the
C-ABI it must give exactly the sum of opl_reduce_sum_f32 (same kernels, same
fixed summation order, so bit-identical) and stay within the reduce gate
(1e-6 relative) of the CPU oracle's FP64 sum.  The calls run back to back on
one stream, a small input first and then larger ones, so that a slot left
unwritten by a later call would still hold the earlier call's partial and
show up as a wrong sum.  This file is collected last so a
stop-at-first-failure run has done everything else.
"""
from __future__ import annotations

import numpy as np
import pytest

import operatorlib
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def test_noalloc_matches_allocating_entry_point_and_oracle(cuda):
    import torch

    lib = operatorlib.capi()
    stream = torch.cuda.Stream(cuda)
    handle = stream.cuda_stream
    rng = np.random.default_rng(2024)
    # Small before large: the larger calls use more scratch slots than the
    # first one wrote.  The last size loops grid-stride (more than 4096 CTAs'
    # worth of single-pass work).
    for n in (1_000_003, 16_777_216, 3, 140_000_001):
        host = rng.uniform(-1, 1, n).astype(np.float32)
        x = torch.from_numpy(host).to(cuda)
        torch.cuda.synchronize()
        got = torch.empty((), device=cuda)
        want = torch.empty((), device=cuda)
        assert lib.opl_reduce_sum_f32_noalloc(x.data_ptr(), got.data_ptr(), n, handle) == 0
        assert lib.opl_reduce_sum_f32(x.data_ptr(), want.data_ptr(), n, handle) == 0
        stream.synchronize()
        g, w = got.item(), want.item()
        assert np.float32(g).tobytes() == np.float32(w).tobytes(), (n, g, w)
        ref = orc.reduce_sum(host)
        assert abs(g - ref) <= 1e-6 * abs(ref) + 1e-6, (n, g, ref)
        del x


def test_noalloc_rejects_bad_arguments():
    lib = operatorlib.capi()
    assert lib.opl_reduce_sum_f32_noalloc(None, 0x1000, 10, None) == 1
    assert lib.opl_reduce_sum_f32_noalloc(0x1000, 0x1000, 0, None) == 1
