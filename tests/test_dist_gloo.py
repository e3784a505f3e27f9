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


def _row_exchange_worker(rank, world, port, out_q):
    """One rank of the row-sharded exchange on CPU: its batch's plan (the
    numpy restatement of engram_shard_plan), every rank's counts gathered
    (NcclRowExchange.gather_counts), ids out and rows back
    (NcclRowExchange.rows, all-to-alls), each owner serving only rows it owns."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from cases import shard_plan_ref
        from engraft_ngram_b200.shard import NcclRowExchange
        from oracle import oracle as O
        n_rows, stride, T = 50_021, 144, 3000
        rng = np.random.default_rng(7)  # the table, its addressing and the overlay: the same on every rank
        full = rng.integers(0, 256, size=(n_rows, stride), dtype=np.uint8)
        sizes = [n_rows // 16 - 3 * (15 - h) for h in range(16)]
        sizes[-1] += n_rows - sum(sizes)
        offs = np.concatenate([[0], np.cumsum(sizes)[:-1]])
        mult = [int(x) | 1 for x in rng.integers(1, 2**63, size=3, dtype=np.uint64)]
        ranks = np.arange(1, 151_937, dtype=np.float64)
        cdf = np.cumsum(ranks ** -1.1)
        cdf /= cdf[-1]
        toks = np.searchsorted(cdf, np.random.default_rng(100 + rank).random(T)).astype(np.int32)
        ids = O.hash_ids(toks, 3, 8, mult, sizes, offs, 151_935)
        ov_ids = np.unique(O.hash_ids(np.searchsorted(cdf, rng.random(T)).astype(np.int32), 3, 8, mult, sizes, offs,
                                      151_935)[::5].reshape(-1))
        send, counts, rix = shard_plan_ref(ids, ov_ids, world, rank)

        class Shard:  # the owner side of the exchange: serves only the rows this rank holds
            def __init__(self):
                self.world, self.rank, self.stride, self.served = world, rank, stride, 0

            def serve(self, recv_ids):
                g = recv_ids.numpy().astype(np.int64)
                assert (g % world == rank).all(), "an owner was asked for a row it does not hold"
                self.served += len(g)
                return torch.from_numpy(full[g].reshape(-1).copy())

        table = Shard()
        ex = NcclRowExchange()
        allc = ex.gather_counts(table, torch.from_numpy(counts)).reshape(world, world).numpy()
        ok = bool((allc[rank] == counts).all()) and allc[rank, rank] == 0
        sc = [int(x) for x in allc[rank]]
        rc = [int(x) for x in allc[:, rank]]
        rows = ex.rows(table, torch.from_numpy(send), sc, rc).numpy().reshape(-1, stride)
        ok &= rows.shape[0] == len(send) and bool((rows == full[send.astype(np.int64)]).all())
        ok &= table.served == sum(rc)
        # every (position, head) finds its row: the overlay, its own shard, or the reply at row_index
        flat = ids.reshape(-1).astype(np.int64)
        req = rix >= 0
        ok &= bool((rows[rix[req]] == full[flat[req]]).all())
        rest = flat[~req]
        ok &= bool(((rest % world == rank) | np.isin(rest, ov_ids)).all())
        remote_pairs = int(((flat % world != rank) & ~np.isin(flat, ov_ids)).sum())
        out_q.put((rank, ok, len(send), remote_pairs))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_row_sharded_exchange_protocol_on_cpu_ranks(world):
    """world gloo ranks on CPU: owner = id mod world, each rank's distinct remote
    rows grouped by owner, the gathered counts matrix, the id and row
    all-to-alls with split sizes from that matrix, and the row index of every
    (position, head) agree with the single-process resident table; a Zipf
    batch requests fewer distinct rows than remote pairs."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_row_exchange_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        rank, ok, distinct, pairs = q.get(timeout=240)
        res[rank] = (ok, distinct, pairs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(v[0] for v in res.values()), res
    assert all(0 < v[1] < v[2] for v in res.values()), res


def _pushed_exchange_worker(rank, world, port, bufs, out_q):
    """One rank of the pushed row exchange on CPU.  Each rank's request buffer,
    count array and send buffer are shared-memory tensors every process maps
    (standing in for torch symmetric memory); the route and the serve follow
    the contracts of engram_shard_route_push / engram_shard_serve_pushed
    (numpy restatements), gloo barriers order them as the exchange's barrier
    does, and the rows come back through the library's own fetch
    (_PushExchange.fetch: one copy per owner from this rank's region of the
    owner's send buffer)."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import types
        from cases import shard_route_push_ref
        from engraft_ngram_b200.shard import _PushExchange
        from oracle import oracle as O
        n_rows, stride, T, nh = 50_021, 144, 3000, 16
        rng = np.random.default_rng(7)  # the table, its addressing and the overlay: the same on every rank
        full = rng.integers(0, 256, size=(n_rows, stride), dtype=np.uint8)
        sizes = [n_rows // 16 - 3 * (15 - h) for h in range(16)]
        sizes[-1] += n_rows - sum(sizes)
        offs = np.concatenate([[0], np.cumsum(sizes)[:-1]])
        mult = [int(x) | 1 for x in rng.integers(1, 2**63, size=3, dtype=np.uint64)]
        ranks = np.arange(1, 151_937, dtype=np.float64)
        cdf = np.cumsum(ranks ** -1.1)
        cdf /= cdf[-1]
        toks = np.searchsorted(cdf, np.random.default_rng(200 + rank).random(T)).astype(np.int32)
        ids = O.hash_ids(toks, 3, 8, mult, sizes, offs, 151_935)
        ov_ids = np.unique(O.hash_ids(np.searchsorted(cdf, rng.random(T)).astype(np.int32), 3, 8, mult, sizes, offs,
                                      151_935)[::5].reshape(-1))
        region = T * nh
        requests, counts, rix = shard_route_push_ref(ids, ov_ids, world, rank)
        # route: each id into region `rank` of its owner's request buffer, the count into its count array
        for o in range(world):
            if o != rank:
                c = int(counts[o])
                bufs[o]["ids"][rank * region:rank * region + c] = torch.from_numpy(requests[o])
                bufs[o]["cnts"][rank] = c
        dist.barrier()  # every rank's route before any owner's serve
        mine = bufs[rank]
        served = 0
        ok = True
        for r in range(world):  # serve: requester r's rows into region r of this owner's send buffer
            if r == rank:
                continue
            c = int(mine["cnts"][r])
            g = mine["ids"][r * region:r * region + c].numpy().astype(np.int64)
            ok &= bool((g % world == rank).all())
            send = mine["send"].view(world * region, stride)
            send[r * region:r * region + c] = torch.from_numpy(full[g])
            served += c
        dist.barrier()  # every owner's serve before any fetch

        class CpuExchange(_PushExchange):
            def _send_rows(self, b, o):
                return bufs[o]["send"]

        table = types.SimpleNamespace(world=world, rank=rank, stride=stride, n_heads=nh, device=torch.device("cpu"))
        ex = CpuExchange()
        ex._setup(table, T, 1)
        rows = ex.fetch(table, 0, [int(x) for x in counts]).numpy().reshape(-1, stride)
        flat = ids.reshape(-1).astype(np.int64)
        req = rix >= 0
        ok &= rows.shape[0] == int(counts.sum()) and counts[rank] == 0
        ok &= bool((rows[rix[req]] == full[flat[req]]).all())  # every requested pair finds its own row
        rest = flat[~req]
        ok &= bool(((rest % world == rank) | np.isin(rest, ov_ids)).all())
        ok &= np.array_equal(np.sort(rix[req]), np.arange(int(req.sum())))
        dist.barrier()
        out_q.put((rank, bool(ok), int(req.sum()), served))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_pushed_row_exchange_bookkeeping_on_cpu_ranks(world):
    """world gloo ranks on CPU with shared-memory buffers: the pushed exchange's
    regions (requester r writes region r of each owner's buffers), per-owner
    counts, the fetch's per-owner offsets and every pair's receive row give
    each rank exactly the rows of its remote, non-overlay pairs; each owner
    serves only rows it holds, and what all owners serve equals what all
    requesters asked for."""
    T, nh, stride = 3000, 16, 144
    region = T * nh
    bufs = [{"ids": torch.full((world * region,), -1, dtype=torch.int32).share_memory_(),
             "cnts": torch.zeros(world, dtype=torch.int64).share_memory_(),
             "send": torch.zeros(world * region * stride, dtype=torch.uint8).share_memory_()} for _ in range(world)]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_pushed_exchange_worker, args=(r, world, port, bufs, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        rank, ok, asked, served = q.get(timeout=240)
        res[rank] = (ok, asked, served)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(v[0] for v in res.values()), res
    assert sum(v[1] for v in res.values()) == sum(v[2] for v in res.values()) > 0
