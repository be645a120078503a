"""Multi-GPU host logic, run as world_size-2 gloo ranks on CPU.

Covers what bench.py does across ranks without needing GPUs: the contiguous
balanced sharding of heads / M blocks / chunks (shard_range), the
max-over-ranks timing reduction, and the reduce path's combine -- per-rank
FP64 partials of contiguous chunks all-reduced in FP64 -- which must equal the
single-process double sum within the 1e-6 gate.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import bench
from oracle import oracle as orc


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port),
                      RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    d = bench.Dist()
    dist.init_process_group("gloo", rank=rank, world_size=world)
    d.pg = dist
    try:
        # max over ranks
        results[f"max{rank}"] = d.max(float(rank + 1) * 1.5)
        # reduce combine: each rank sums its chunk in FP64, then all-reduce
        x = np.random.default_rng(7).uniform(-1, 1, 1_000_003).astype(np.float32)
        lo, hi = bench.shard_range(x.size, world, rank)
        part = torch.tensor([orc.reduce_sum(x[lo:hi])], dtype=torch.float64)
        dist.all_reduce(part)
        results[f"sum{rank}"] = float(part.item())
        d.barrier()
    finally:
        dist.destroy_process_group()


def test_shard_range_covers_everything_once():
    for total in (0, 1, 7, 256, 16384, 1_000_003):
        for world in (1, 2, 3, 4, 8):
            spans = [bench.shard_range(total, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
                assert a1 == b0
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1


@pytest.mark.timeout(120)
def test_two_rank_gloo_reduce_combine_and_max():
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(100)
        assert p.exitcode == 0
    assert results["max0"] == results["max1"] == 3.0
    x = np.random.default_rng(7).uniform(-1, 1, 1_000_003).astype(np.float32)
    want = orc.reduce_sum(x)
    for r in range(2):
        assert abs(results[f"sum{r}"] - want) <= 1e-6 * abs(want)
