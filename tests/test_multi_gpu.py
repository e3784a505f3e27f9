"""Multi-GPU paths on real ranks (one process per GPU, NCCL).  Skipped with
fewer than two GPUs; the single-GPU suite covers the same kernels with ranks
emulated on one device."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


# Every rank runs with NVLS off in NCCL and with torch's symmetric memory mapped
# without an NVLink multicast object; no kernel here waits on another GPU, and
# the process group's short timeout ends a rank whose peer stops answering.
RANK_ENV = dict(MASTER_ADDR="127.0.0.1", NCCL_NVLS_ENABLE="0", TORCH_SYMM_MEM_DISABLE_MULTICAST="1")
PG_TIMEOUT_S = 60


def _run_ranks(target, world: int = 2) -> dict:
    """Runs target(rank, world, port, out) in `world` spawned processes and
    returns out.  A rank is never killed: each one ends by itself, at the
    latest when a collective of its process group times out."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, out), daemon=True) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=20 * PG_TIMEOUT_S)
    alive = [p.pid for p in procs if p.is_alive()]
    assert not alive, f"ranks still running after {20 * PG_TIMEOUT_S} s: {alive}"
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    return dict(out)


def _peer_vs_nccl(rank: int, world: int, port: int, out) -> None:
    import torch.distributed as dist
    from datetime import timedelta
    os.environ.update(RANK_ENV, MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=PG_TIMEOUT_S), device_id=dev)
    try:
        import engraft_ngram_b200 as eb
        from engraft_ngram_b200 import _lib as L
        from engraft_ngram_b200.dist import PeerRows, all_gather_rows, reduce_scatter_rows, shard_bounds
        R, dim, T, nh, hpn = 4000, 256, 2048, 16, 8
        mode = L.MODE_PAIRSUM_ADD_BF16
        rng = np.random.default_rng(5)
        p_init = torch.from_numpy((rng.standard_normal((R, dim)) * 0.01).astype(np.float32)).to(dev)
        lo, hi = shard_bounds(R, world, rank)
        peer = PeerRows(R, dim, dev)
        peer.rows_var.copy_(p_init)
        m1, v1 = torch.zeros(hi - lo, dim, device=dev), torch.zeros(hi - lo, dim, device=dev)
        rows2 = p_init.clone()
        m2, v2 = torch.zeros(hi - lo, dim, device=dev), torch.zeros(hi - lo, dim, device=dev)
        rr = np.random.default_rng(100 + rank)  # each rank its own batch
        ok = True
        for step in (1, 2, 3):
            slots = np.full((T, nh), -1, dtype=np.int32)
            hit = rr.random((T, nh)) < 0.3
            slots[hit] = rr.integers(0, R, size=int(hit.sum()))
            sl = torch.from_numpy(slots).to(dev)
            g = torch.from_numpy((rr.standard_normal((T, hpn * dim)) * 1e-2).astype(np.float32)).to(dev).to(
                torch.bfloat16)
            peer.backward(sl, g, nh, hpn, mode)
            peer.step(m1, v1, p_init[lo:hi], step, 1e-3, reg_scale=0.25)
            shard = reduce_scatter_rows(eb.row_gradients(sl, g, nh, hpn, dim, R, mode))
            p = rows2[lo:hi]
            st = L.load().engram_adam_step(p.data_ptr(), shard.data_ptr(), m2.data_ptr(), v2.data_ptr(),
                                           p_init[lo:hi].data_ptr(), p.numel(), step, 1e-3, 0.9, 0.999, 1e-8, 0.25,
                                           L.stream_of(dev))
            L.check(st, "engram_adam_step")
            all_gather_rows(rows2, p)
            torch.cuda.synchronize()
            ok &= torch.equal(peer.rows_var.view(torch.int32), rows2.view(torch.int32))
            ok &= torch.equal(m1.view(torch.int32), m2.view(torch.int32))
        out[rank] = bool(ok)
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_peer_exchange_matches_nccl_collectives_on_two_ranks():
    """Two ranks: backward into the owners' buffers + the owner step equal the
    dense backward + NCCL reduce-scatter + Adam + all-gather bit for bit (a
    two-term sum does not depend on order)."""
    assert _run_ranks(_peer_vs_nccl) == {0: True, 1: True}


def _sharded_staging(rank: int, world: int, port: int, out) -> None:
    """Each rank: its shard in symmetric memory; three batches run through the
    prefetch-then-forward pipeline with push staging and with pull staging, and
    once read in place; every output equals the forward over the whole
    resident table."""
    import ctypes as C
    import torch.distributed as dist
    from datetime import timedelta
    os.environ.update(RANK_ENV, MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=PG_TIMEOUT_S), device_id=dev)
    try:
        import engraft_ngram_b200 as eb
        from engraft_ngram_b200 import _lib as L
        from engraft_ngram_b200.shard import ShardedTable, peer_shard_buffer
        from engraft_ngram_b200.table import synthetic_head_sizes, synthetic_multipliers, synthetic_resident
        n_rows, fmt, dim, T, eos = 60_013, L.FMT_NAMES["iq4_xs"], 256, 1500, 151_935
        mode = L.MODE_PAIRSUM_ADD_BF16
        sizes = synthetic_head_sizes(n_rows)
        offs = np.concatenate([[0], np.cumsum(sizes)[:-1]]).tolist()
        mult = synthetic_multipliers(4)
        full = eb.DeviceTable(synthetic_resident(n_rows, fmt, dim, 11, dev), fmt, dim, sizes, offs, mult, eos,
                              n_rows=n_rows)
        stride = full.row_stride
        buf, ptrs, _h = peer_shard_buffer(n_rows, fmt, dim, dev)
        mine = full.rows.view(n_rows, stride)[rank::world].reshape(-1)
        buf[: mine.numel()].copy_(mine)
        torch.cuda.synchronize()
        dist.barrier()
        push = ShardedTable(buf, fmt, dim, sizes, offs, mult, eos, world, rank, n_rows, peer_ptrs=ptrs)
        push.enable_push_staging(T)
        pull = ShardedTable(buf, fmt, dim, sizes, offs, mult, eos, world, rank, n_rows, peer_ptrs=ptrs)
        rng = np.random.default_rng(9)  # the overlay is the same on every rank
        ov_ids = np.unique(rng.integers(0, n_rows, size=3000)).astype(np.int32)
        omap = eb.OverlayMap(torch.from_numpy(ov_ids), dev)
        rows_var = torch.from_numpy((rng.standard_normal((len(ov_ids), dim)) * 0.01).astype(np.float32)).to(dev)
        ranks = np.arange(1, 151_937, dtype=np.float64)
        cdf = np.cumsum(ranks ** -1.1)
        cdf /= cdf[-1]
        rr = np.random.default_rng(200 + rank)  # each rank its own batches
        batches = []
        for _ in range(3):
            toks = np.searchsorted(cdf, rr.random(T)).astype(np.int32)
            seg = np.sort(rr.integers(0, 3, size=T))
            ss = np.concatenate([[0], np.flatnonzero(np.diff(seg)) + 1])
            starts = np.repeat(ss, np.diff(np.concatenate([ss, [T]]))).astype(np.int32)
            batches.append((torch.from_numpy(toks).to(dev), torch.from_numpy(starts).to(dev)))
        res0 = (torch.from_numpy(rr.standard_normal((T, 8 * dim)).astype(np.float32)) * 0.5).to(dev).to(torch.bfloat16)

        def resident(tok, ss):
            out = res0.clone()
            ov = omap.descriptor(rows_var)
            st = L.load().engram_forward(C.byref(full.ctable), C.byref(ov), tok.data_ptr(), ss.data_ptr(), 0, T, mode,
                                         out.data_ptr(), None, None, None, L.stream_of(dev))
            L.check(st, "engram_forward")
            return out

        ok = True
        for table in (push, pull):
            table.prefetch(*batches[0], omap=omap)
            for k in range(3):
                if k + 1 < 3:
                    table.prefetch(*batches[k + 1], omap=omap)
                got = res0.clone()
                table.forward(batches[k][0], batches[k][1], omap, rows_var, got, mode)
                ok &= torch.equal(got.view(torch.int16), resident(*batches[k]).view(torch.int16))
        got = res0.clone()
        pull.forward(batches[1][0], batches[1][1], omap, rows_var, got, mode)  # not prefetched: read in place
        ok &= torch.equal(got.view(torch.int16), resident(*batches[1]).view(torch.int16))
        torch.cuda.synchronize()
        dist.barrier()
        out[rank] = bool(ok)
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_row_sharded_staging_matches_resident_table_on_two_ranks():
    """Two ranks, table row-sharded in symmetric memory: push-staged,
    pull-staged and in-place sharded forwards equal the resident-table forward
    bit for bit, over three pipelined batches."""
    assert _run_ranks(_sharded_staging) == {0: True, 1: True}


def _autograd_peer(rank: int, world: int, port: int, out) -> None:
    """Each rank: three steps through the public autograd API on its own batch,
    once with the row gradients routed into PeerRows (attach + PeerAdam) and
    once with the NCCL all-reduce of rows_var.grad + OverlayAdam; the rows and
    the hit counts agree bit for bit."""
    import torch.distributed as dist
    from datetime import timedelta
    os.environ.update(RANK_ENV, MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=PG_TIMEOUT_S), device_id=dev)
    try:
        import engraft_ngram_b200 as eb
        from engraft_ngram_b200 import _lib as L
        from engraft_ngram_b200.dist import PeerAdam, PeerRows
        from engraft_ngram_b200.table import synthetic_head_sizes, synthetic_multipliers, synthetic_resident
        n_rows, fmt, dim, T, eos = 70_001, L.FMT_NAMES["iq4_xs"], 256, 1200, 151_935
        sizes = synthetic_head_sizes(n_rows)
        offs = np.concatenate([[0], np.cumsum(sizes)[:-1]]).tolist()
        table = eb.DeviceTable(synthetic_resident(n_rows, fmt, dim, 21, dev), fmt, dim, sizes, offs,
                               synthetic_multipliers(6), eos, n_rows=n_rows)
        ranks = np.arange(1, 151_937, dtype=np.float64)
        cdf = np.cumsum(ranks ** -1.1)
        cdf /= cdf[-1]
        rr = np.random.default_rng(300 + rank)
        batches = [torch.from_numpy(np.searchsorted(cdf, rr.random(T)).astype(np.int32)).to(dev) for _ in range(3)]
        g0 = np.random.default_rng(8)  # overlay ids, start rows and residual: the same on every rank
        shared = torch.from_numpy(np.searchsorted(cdf, g0.random(T)).astype(np.int32)).to(dev)
        ids = table.global_ids(shared).reshape(-1)
        ov_ids = torch.unique(torch.cat([ids[::3], torch.from_numpy(g0.integers(0, n_rows, 500)).to(dev).int()]))
        R = int(ov_ids.numel())
        p0 = torch.from_numpy((g0.standard_normal((R, dim)) * 0.01).astype(np.float32)).to(dev)
        res0 = torch.from_numpy((g0.standard_normal((T, 8 * dim)) * 0.5).astype(np.float32)).to(dev).to(torch.bfloat16)
        dout = torch.from_numpy((rr.standard_normal((T, 8 * dim)) * 1e-3).astype(np.float32)).to(dev).to(torch.bfloat16)

        def run(peer_mode: bool):
            omap = eb.OverlayMap(ov_ids, dev)
            hits = torch.zeros(3, dtype=torch.int64, device=dev)
            if peer_mode:
                peer = PeerRows(R, dim, dev)
                peer.rows_var.copy_(p0)
                rows_var = peer.rows_var.requires_grad_(True)
                peer.attach(omap)
                opt = PeerAdam(peer, lr=1e-3, reg_ref=p0, reg_mu=0.1)
            else:
                rows_var = p0.clone().requires_grad_(True)
                opt = eb.OverlayAdam([rows_var], lr=1e-3, reg_ref=p0, reg_mu=0.1)
            for k in range(3):
                opt.zero_grad()
                o = eb.engram_residual_add(res0.clone(), table, batches[k], rows_var, omap, None, 0, hits[k:k + 1])
                o.backward(dout)
                if not peer_mode:
                    assert rows_var.grad is not None
                    dist.all_reduce(rows_var.grad)
                else:
                    assert rows_var.grad is None
                opt.step()
            torch.cuda.synchronize()
            return rows_var.detach().clone(), hits

        a, ha = run(True)
        b, hb = run(False)
        out[rank] = bool(torch.equal(a.view(torch.int32), b.view(torch.int32)) and torch.equal(ha, hb))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_autograd_through_peer_rows_matches_allreduce_on_two_ranks():
    """Two ranks, public autograd API: PeerRows.attach + PeerAdam equals the
    NCCL all-reduce of the row gradients + OverlayAdam bit for bit."""
    assert _run_ranks(_autograd_peer) == {0: True, 1: True}


def _exchange_staging(rank: int, world: int, port: int, out) -> None:
    """Each rank: its shard in plain local memory and exchange staging (the
    default peer exchange: requests pushed into the owners' symmetric memory,
    owners gather locally, requesters copy with the copy engines; then the
    NCCL all-to-all exchange); four batches, the last two forwarded with
    stages still to run, each forward equal bit for bit to the resident-table
    forward of the same batch."""
    import ctypes as C
    import torch.distributed as dist
    from datetime import timedelta
    os.environ.update(RANK_ENV, MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=PG_TIMEOUT_S), device_id=dev)
    try:
        import engraft_ngram_b200 as eb
        from engraft_ngram_b200 import _lib as L
        from engraft_ngram_b200.shard import ShardedTable
        from engraft_ngram_b200.table import synthetic_head_sizes, synthetic_multipliers, synthetic_resident
        n_rows, fmt, dim, T, eos = 60_013, L.FMT_NAMES["iq4_xs"], 256, 1500, 151_935
        mode = L.MODE_PAIRSUM_ADD_BF16
        sizes = synthetic_head_sizes(n_rows)
        offs = np.concatenate([[0], np.cumsum(sizes)[:-1]]).tolist()
        mult = synthetic_multipliers(4)
        full = eb.DeviceTable(synthetic_resident(n_rows, fmt, dim, 11, dev), fmt, dim, sizes, offs, mult, eos,
                              n_rows=n_rows)
        ok = True
        for exchange in ("peer", "nccl"):
            sh = ShardedTable.from_full(full, world, rank)
            sh.enable_exchange_staging(T, exchange)
            rng = np.random.default_rng(9)  # the overlay is the same on every rank
            ov_ids = np.unique(rng.integers(0, n_rows, size=3000)).astype(np.int32)
            omap = eb.OverlayMap(torch.from_numpy(ov_ids), dev)
            rows_var = torch.from_numpy((rng.standard_normal((len(ov_ids), dim)) * 0.01).astype(np.float32)).to(dev)
            ranks = np.arange(1, 151_937, dtype=np.float64)
            cdf = np.cumsum(ranks ** -1.1)
            cdf /= cdf[-1]
            rr = np.random.default_rng(400 + rank)  # each rank its own batches
            batches = []
            for _ in range(4):
                toks = np.searchsorted(cdf, rr.random(T)).astype(np.int32)
                seg = np.sort(rr.integers(0, 3, size=T))
                ss = np.concatenate([[0], np.flatnonzero(np.diff(seg)) + 1])
                starts = np.repeat(ss, np.diff(np.concatenate([ss, [T]]))).astype(np.int32)
                batches.append((torch.from_numpy(toks).to(dev), torch.from_numpy(starts).to(dev)))
            res0 = (torch.from_numpy(rr.standard_normal((T, 8 * dim)).astype(np.float32)) * 0.5).to(dev).to(
                torch.bfloat16)

            def resident(tok, ss):
                o = res0.clone()
                ov = omap.descriptor(rows_var)
                st = L.load().engram_forward(C.byref(full.ctable), C.byref(ov), tok.data_ptr(), ss.data_ptr(), 0, T,
                                             mode, o.data_ptr(), None, None, None, L.stream_of(dev))
                L.check(st, "engram_forward")
                return o

            sh.prefetch(*batches[0], omap=omap)
            sh.prefetch(*batches[1], omap=omap)
            for k in range(4):
                if k + 2 < 4:
                    sh.prefetch(*batches[k + 2], omap=omap)
                got = res0.clone()
                sh.forward(batches[k][0], batches[k][1], omap, rows_var, got, mode)
                ok &= torch.equal(got.view(torch.int16), resident(*batches[k]).view(torch.int16))
            torch.cuda.synchronize()
        dist.barrier()
        out[rank] = bool(ok)
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_exchange_staging_matches_resident_table_on_two_ranks():
    """Two ranks, table row-sharded in local memory: the exchange staged ahead
    of the forward, over peer memory (pushed requests, copy-engine transfers)
    and over NCCL all-to-alls, feeds forwards bit-identical to the
    resident-table forward."""
    assert _run_ranks(_exchange_staging) == {0: True, 1: True}
