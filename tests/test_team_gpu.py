"""Fused multi-GPU reduce (opl_team_*): each rank sums its contiguous chunk
and the partials are combined over NVLink peer memory inside the reduce's
own kernels.  Runs as child processes on 2 GPUs (skipped with fewer): every
rank must get the bit-identical total, within 1e-6 of the FP64 sum of the
whole array, over repeated calls (call counter and slot parity advance) and
over CUDA-graph replays of one captured call."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q):
    import sys

    import torch
    import torch.distributed as dist

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [os.path.join(root, "orin-cuda-operator-library_b200"), root]
    import bench
    import operatorlib
    from oracle import oracle as orc

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        team = operatorlib.ReduceTeam(rank, world)
        out = torch.empty((), device="cuda")
        results = []
        for call, n in enumerate([1_000_003, 16_777_216, 7, 4_194_304, 999]):
            x = np.random.default_rng(100 + call).uniform(-1, 1, n).astype(np.float32)
            lo, hi = bench.shard_range(n, world, rank)
            chunk = torch.from_numpy(x[lo:hi].copy() if hi > lo else np.zeros(1, np.float32)).cuda()
            if hi == lo:  # an empty chunk contributes an exact 0.0 partial
                chunk.zero_()
            team.reduce_sum_into(chunk, out)
            torch.cuda.synchronize()
            results.append((out.item(), orc.reduce_sum(x)))
        # back-to-back calls alternating two inputs of the same size: a
        # finalize that read its partials before the partial kernel wrote
        # them would pick up the other input's (same workspace memory)
        xa = np.random.default_rng(11).uniform(-1, 1, 16_777_216).astype(np.float32)
        xb = np.random.default_rng(12).uniform(-1, 1, 16_777_216).astype(np.float32)
        lo, hi = bench.shard_range(xa.size, world, rank)
        ca, cb = (torch.from_numpy(v[lo:hi].copy()).cuda() for v in (xa, xb))
        outs = torch.empty(6, device="cuda")
        for k in range(6):
            team.reduce_sum_into(ca if k % 2 == 0 else cb, outs[k])
        torch.cuda.synchronize()
        for k in range(6):
            results.append((outs[k].item(), orc.reduce_sum(xa if k % 2 == 0 else xb)))
        # one captured call replayed three times
        x = np.random.default_rng(7).uniform(-1, 1, 2_000_000).astype(np.float32)
        lo, hi = bench.shard_range(x.size, world, rank)
        chunk = torch.from_numpy(x[lo:hi].copy()).cuda()
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                team.launch(chunk, out, s.cuda_stream)
        for _ in range(3):
            g.replay()
            torch.cuda.synchronize()
            results.append((out.item(), orc.reduce_sum(x)))
        code = __import__("ctypes").c_int(0)
        operatorlib.capi().opl_read_and_clear_watchdog(code)
        team.close()
        q.put((rank, results, code.value))
    finally:
        dist.destroy_process_group()


def test_team_reduce_two_gpus():
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(world):
        rank, results, code = q.get(timeout=240)
        got[rank] = (results, code)
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    assert got[0][1] == 0 and got[1][1] == 0, "watchdog tripped"
    for (a, want), (b, _) in zip(got[0][0], got[1][0]):
        assert a == b  # bit-identical on every rank
        assert abs(a - want) <= 1e-6 * abs(want) + 1e-6, (a, want)
