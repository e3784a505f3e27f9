"""ExchangeStage's staging protocol on CPU, for the pushing exchange: the CUDA
stream and event objects are replaced by recording stand-ins and the exchange
by one that logs its calls, so the order of route, serve, barrier and fetch
that every rank issues can be checked without a GPU.  The data path is checked
on the GPU (tests/test_gpu_parity.py, tests/test_multi_gpu.py); this pins the
sequencing those tests rely on."""
from __future__ import annotations

import contextlib
import itertools

import pytest
import torch

from engraft_ngram_b200 import shard as S

_ids = itertools.count()


class FakeStream:
    def __init__(self, *a, **k):
        self.cuda_stream = next(_ids)

    def wait_event(self, ev):
        pass

    def wait_stream(self, s):
        pass


class FakeEvent:
    def __init__(self, *a, **k):
        pass

    def record(self, stream=None):
        pass

    def synchronize(self):
        pass

    def elapsed_time(self, other):
        return 0.0


@pytest.fixture
def fake_cuda(monkeypatch):
    cur = {"s": FakeStream()}

    @contextlib.contextmanager
    def stream(s):
        prev = cur["s"]
        cur["s"] = s
        try:
            yield
        finally:
            cur["s"] = prev

    monkeypatch.setattr(torch.cuda, "Stream", FakeStream)
    monkeypatch.setattr(torch.cuda, "Event", FakeEvent)
    monkeypatch.setattr(torch.cuda, "current_stream", lambda device=None: cur["s"])
    monkeypatch.setattr(torch.cuda, "stream", stream)
    monkeypatch.setattr(torch.Tensor, "pin_memory", lambda self: self)
    monkeypatch.setattr(torch.Tensor, "record_stream", lambda self, s: None)
    return cur


class Table:
    def __init__(self, world, rank):
        self.world, self.rank, self.n_heads, self.stride, self.device = world, rank, 16, 144, torch.device("cpu")


class LoggingExchange:
    """A pushing exchange that records (call, rank, set, batch) for every call."""
    pushes = True

    def __init__(self, log, rank, world):
        self.log, self.rank, self.world = log, rank, world
        self.batch_of_set = {}

    def route(self, table, b, ov, tokens, ss, t0, n, counts, row_index, stream):
        batch = int(tokens[0])
        self.batch_of_set[b] = batch
        counts[: self.world] = torch.tensor([0 if o == self.rank else 1 for o in range(self.world)])
        self.log.append(("route", self.rank, b, batch))

    def serve(self, table, b):
        self.log.append(("serve", self.rank, b, self.batch_of_set[b]))

    def barrier(self):
        self.log.append(("barrier", self.rank, None, None))

    def fetch(self, table, b, own):
        self.log.append(("fetch", self.rank, b, self.batch_of_set[b]))
        return torch.full((sum(own) * table.stride,), self.batch_of_set[b] % 251, dtype=torch.uint8)


def _drive(world, batches, depth, unprefetched=0):
    """Every rank prefetches `depth` batches ahead and forwards in order, as
    real ranks do; the last `unprefetched` batches are forwarded without a
    prefetch (ShardedTable.forward's path: prefetch on the spot, then take)."""
    log = []
    stages = []
    for r in range(world):
        ex = LoggingExchange(log, r, world)
        stages.append(S.ExchangeStage(Table(world, r), 4096, ex))
    toks = [torch.full((64,), k, dtype=torch.int32) for k in range(batches)]
    taken = {}

    def pre(r, k):
        stages[r].prefetch(("batch", k), toks[k], None, 0, 64, None)

    last_pref = batches - unprefetched
    for k in range(min(depth, last_pref)):
        for r in range(world):
            pre(r, k)
    for k in range(batches):
        for r in range(world):
            if k + depth < last_pref:
                pre(r, k + depth)
        for r in range(world):
            st = stages[r]
            if not st.has(("batch", k)):
                pre(r, k)
            b, recv, rix, ready = st.take(("batch", k), None)
            taken[(r, k)] = (b, int(recv[0]) if recv.numel() else None)
            st.consumed(b, torch.cuda.current_stream())
    return log, taken


def _per_rank(log, rank):
    return [e for e in log if e[1] == rank]


@pytest.mark.parametrize("world,batches,depth,unprefetched", [(2, 8, 3, 0), (3, 9, 3, 2), (2, 6, 2, 1)])
def test_pushed_staging_orders_route_serve_fetch_with_barriers_between(fake_cuda, world, batches, depth,
                                                                       unprefetched):
    log, taken = _drive(world, batches, depth, unprefetched)
    for r in range(world):
        ev = _per_rank(log, r)
        pos = {}
        for i, (call, _, b, batch) in enumerate(ev):
            if call != "barrier":
                assert (call, batch) not in pos, (r, call, batch)  # each stage once per batch
                pos[(call, batch)] = (i, b)
        barriers = [i for i, e in enumerate(ev) if e[0] == "barrier"]
        for k in range(batches):
            i_r, b_r = pos[("route", k)]
            i_s, b_s = pos[("serve", k)]
            i_f, b_f = pos[("fetch", k)]
            assert b_r == b_s == b_f  # one buffer set per batch
            assert i_r < i_s < i_f
            # every rank's route is closed by a barrier before any owner serves it, and every serve before any fetch
            assert any(i_r < i < i_s for i in barriers), (r, k)
            assert any(i_s < i < i_f for i in barriers), (r, k)
            assert taken[(r, k)] == (b_r, k % 251)  # the forward reads the set its batch was fetched into
    # every rank issues the same barriers, and each batch has the same set on every rank
    n_bar = {r: sum(1 for e in _per_rank(log, r) if e[0] == "barrier") for r in range(world)}
    assert len(set(n_bar.values())) == 1, n_bar
    for k in range(batches):
        sets = {e[2] for e in log if e[0] == "route" and e[3] == k}
        assert len(sets) == 1, (k, sets)


def test_pushed_staging_keeps_at_most_four_batches(fake_cuda):
    """Five prefetches with no forward: the oldest batch is dropped on every
    rank alike, and the sets stay distinct among the batches kept."""
    log = []
    st = S.ExchangeStage(Table(2, 0), 4096, LoggingExchange(log, 0, 2))
    toks = [torch.full((64,), k, dtype=torch.int32) for k in range(5)]
    for k in range(5):
        st.prefetch(("batch", k), toks[k], None, 0, 64, None)
    assert not st.has(("batch", 0)) and all(st.has(("batch", k)) for k in range(1, 5))
    kept = [st.key.index(("batch", k)) for k in range(1, 5)]
    assert len(set(kept)) == 4
