"""Failure detection of the fused multi-GPU reduce without a GPU fault.

Two processes on one GPU form a 2-rank team (team buffers opened through
CUDA IPC).  Rank 1 connects and then stays idle -- it never launches a
reduce -- while keeping its buffer alive; rank 0 launches opl_team_reduce_sum_f32
alone.  Rank 0's finalize kernel posts its partial, waits (bounded) for a
flag that nothing sets, gives up, writes NaN as the total and records the
watchdog code 0x6e04; the host reads both and the context stays usable.
The timeout is final for the team: the next call on rank 0 posts nothing
and returns NaN at once, without waiting and without a new watchdog code.
Only one rank ever runs a kernel, so no two kernels wait on each other.
"""
from __future__ import annotations

import ctypes
import math
import multiprocessing as mp
import os
import sys
import time

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HANDLE_BYTES = 64  # sizeof(cudaIpcMemHandle_t)
WATCHDOG_TEAM = 0x6E04


def _lib():
    sys.path[:0] = [os.path.join(ROOT, "orin-cuda-operator-library_b200"), ROOT]
    import operatorlib

    return operatorlib, operatorlib.capi()


def _idle_rank(conn):
    """Rank 1: create and connect, then wait until rank 0 is done."""
    import torch

    torch.cuda.set_device(0)
    _, lib = _lib()
    team = ctypes.c_void_p()
    handle = ctypes.create_string_buffer(HANDLE_BYTES)
    rc = lib.opl_team_create(1, 2, ctypes.byref(team), handle)
    conn.send((rc, handle.raw))
    if rc != 0:
        return
    h0 = conn.recv()
    rc = lib.opl_team_connect(team, ctypes.create_string_buffer(h0 + handle.raw, 2 * HANDLE_BYTES))
    conn.send(rc)
    conn.recv()  # rank 0 finished with this rank's buffer
    conn.send(lib.opl_team_destroy(team))


def test_peer_that_never_posts_times_out(cuda):
    import torch

    operatorlib, lib = _lib()
    ctx = mp.get_context("spawn")
    parent, child = ctx.Pipe()
    proc = ctx.Process(target=_idle_rank, args=(child,))
    proc.start()
    try:
        team = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(HANDLE_BYTES)
        assert lib.opl_team_create(0, 2, ctypes.byref(team), handle) == 0
        rc1, h1 = parent.recv()
        assert rc1 == 0
        parent.send(handle.raw)
        both = ctypes.create_string_buffer(handle.raw + h1, 2 * HANDLE_BYTES)
        assert lib.opl_team_connect(team, both) == 0
        assert parent.recv() == 0

        code = ctypes.c_int(0)
        lib.opl_read_and_clear_watchdog(ctypes.byref(code))
        x = torch.ones(10_000, device=cuda)
        out = torch.zeros((), device=cuda)
        stream = torch.cuda.current_stream(cuda)
        rc = lib.opl_team_reduce_sum_f32(team, ctypes.c_void_p(x.data_ptr()),
                                         ctypes.c_void_p(out.data_ptr()), x.numel(),
                                         ctypes.c_void_p(stream.cuda_stream))
        assert rc == 0
        stream.synchronize()  # returns: the wait is bounded
        assert math.isnan(out.item())
        assert lib.opl_read_and_clear_watchdog(ctypes.byref(code)) == 0
        assert code.value == WATCHDOG_TEAM
        # the failed team stays failed: the next call answers NaN at once
        out.zero_()
        t0 = time.monotonic()
        rc = lib.opl_team_reduce_sum_f32(team, ctypes.c_void_p(x.data_ptr()),
                                         ctypes.c_void_p(out.data_ptr()), x.numel(),
                                         ctypes.c_void_p(stream.cuda_stream))
        assert rc == 0
        stream.synchronize()
        assert time.monotonic() - t0 < 1.0  # no second bounded wait
        assert math.isnan(out.item())
        assert lib.opl_read_and_clear_watchdog(ctypes.byref(code)) == 0
        assert code.value == 0
        # the context is still usable
        y = torch.empty((), device=cuda)
        operatorlib.reduce_sum_into(x, y)
        stream.synchronize()
        assert y.item() == 10_000.0
        assert lib.opl_team_destroy(team) == 0
        parent.send("done")
        assert parent.recv() == 0
    finally:
        proc.join(timeout=120)
        if proc.is_alive():
            proc.kill()
    assert proc.exitcode == 0
