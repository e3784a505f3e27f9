"""The multi-rank overlay exchange (reduce-scatter of row gradients, sharded
update, all-gather of rows) run as world_size-2 gloo processes on CPU."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from engraft_ngram_b200.dist import all_gather_rows, reduce_scatter_rows, shard_bounds


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, R, D, out_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.from_numpy(np.random.default_rng(rank).standard_normal((R, D)).astype(np.float32))
        shard = reduce_scatter_rows(g)
        lo, hi = shard_bounds(R, world, rank)
        rows = torch.zeros(R, D)
        upd = shard * 2.0 + rank  # stand-in for the owner's update
        all_gather_rows(rows, upd)
        out_q.put((rank, lo, hi, shard.numpy().copy(), rows.numpy().copy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("R", [40, 41])
def test_reduce_scatter_and_all_gather_two_ranks(R):
    world, D = 2, 8
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, R, D, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        rank, lo, hi, shard, rows = q.get(timeout=120)
        res[rank] = (lo, hi, shard, rows)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    total = sum(np.random.default_rng(r).standard_normal((R, D)).astype(np.float32) for r in range(world))
    expect_rows = np.zeros((R, D), np.float32)
    for r in range(world):
        lo, hi, shard, rows = res[r]
        np.testing.assert_allclose(shard, total[lo:hi], rtol=1e-6, atol=1e-6)
        expect_rows[lo:hi] = shard * 2.0 + r
    for r in range(world):
        np.testing.assert_allclose(res[r][3], expect_rows, rtol=0, atol=0)


def test_shard_bounds_cover_all_rows():
    for R in (0, 1, 7, 40000, 40001):
        for W in (1, 2, 3, 8):
            spans = [shard_bounds(R, W, r) for r in range(W)]
            assert spans[0][0] == 0 and spans[-1][1] == R
            assert all(spans[i][1] == spans[i + 1][0] for i in range(W - 1))
    with pytest.raises(ValueError):
        shard_bounds(10, 2, 2)
