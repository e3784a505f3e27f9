"""Row-sharded resident table across W GPUs: owner(g) = g mod W, local index g / W.

Each rank holds 1/W of the table.  Two ways to read it:
- peer memory (peer_ptrs set): every rank's shard lives in torch symmetric
  memory, so the forward kernels copy each row straight from its owner over
  NVLink (engram_forward_sharded); nothing runs before the forward.  The
  shards never change (training updates the overlay only), so the rows of
  other ranks that a forward will read can be copied ahead, on a side stream
  while the previous step runs (prefetch -> engram_stage_sharded); the
  forward over the same tokens then reads every row from local HBM
  (engram_forward_staged);
- an exchange (NCCL): a rank hashes its positions, skips the heads the overlay
  serves, sends the distinct remaining row ids to their owners (all-to-all-v),
  receives the quantised rows (a second all-to-all-v) into local HBM, and runs
  the forward over those rows (engram_forward_indirect).  The exchange is
  pluggable: `nccl_exchange` for real ranks, or any function with the same
  contract (the tests emulate W ranks on one GPU).
The overlay itself is replicated and updated as in the data-parallel path
(engraft_ngram_b200.dist).
"""
from __future__ import annotations

import ctypes as C
from collections import OrderedDict

import numpy as np
import torch

from . import _lib as L
from .overlay import OverlayMap
from .table import DeviceTable, _as_i32


class ShardedTable:
    def __init__(self, shard_rows: torch.Tensor, fmt: int, dim: int, head_sizes, head_offsets, mult, eos_token_id,
                 world: int, rank: int, n_rows: int, ngram_size: int = 3, heads_per_ngram: int = 8, exchange=None,
                 peer_ptrs: torch.Tensor | None = None):
        """shard_rows: uint8 CUDA tensor with this rank's rows in resident layout
        (global rows rank, rank+W, rank+2W, ... in order).  exchange: the row
        exchange the public API (engram_embed, engram_residual_add) uses with
        this table, e.g. nccl_exchange(); settable later as .exchange.
        peer_ptrs: int64 device tensor [W] of every rank's shard address in
        this process (peer_shard_buffer); when set, forward() reads rows in
        place and needs no exchange."""
        if not (0 <= rank < world):
            raise ValueError(f"rank {rank} of {world}")
        lib = L.load()
        self.fmt, self.dim, self.world, self.rank, self.n_rows = int(fmt), int(dim), int(world), int(rank), int(n_rows)
        self.stride = int(lib.engram_row_stride(fmt, dim))
        self.n_local = (self.n_rows - rank + world - 1) // world
        if shard_rows.numel() < self.n_local * self.stride:
            raise ValueError("shard buffer too small")
        self.shard = shard_rows
        self.device = shard_rows.device
        self.exchange = exchange
        self.peer_ptrs = peer_ptrs
        self.is_sharded = True
        self._staged = OrderedDict()  # prefetch key -> _Staged, waiting for its forward
        self._free = []  # _Staged buffers whose forward has been issued
        self._side = None  # the prefetch stream
        self.push = None  # PushStage: owners copy rows into the requesters' stages (enable_push_staging)
        self.xstage = None  # ExchangeStage: deduplicated rows exchanged ahead of the forward (enable_exchange_staging)
        # addressing constants of the whole table; the rows pointer is replaced per step
        self.ngram_size, self.heads_per_ngram = int(ngram_size), int(heads_per_ngram)
        self.n_heads = (int(ngram_size) - 1) * int(heads_per_ngram)
        sizes = np.asarray([int(x) for x in head_sizes], dtype=np.int64)
        offs = np.asarray([int(x) for x in head_offsets], dtype=np.int64)
        mu = np.asarray([int(m) & 0xFFFFFFFFFFFFFFFF for m in mult], dtype=np.uint64)
        self.ctable = L.EngramTable()
        st = lib.engram_table_init(C.byref(self.ctable), shard_rows.data_ptr(), self.n_rows, self.fmt, self.dim,
                                   int(ngram_size), int(heads_per_ngram), sizes.ctypes.data, offs.ctypes.data,
                                   mu.ctypes.data, len(mu), int(eos_token_id))
        L.check(st, "engram_table_init")

    @classmethod
    def from_full(cls, full: DeviceTable, world: int, rank: int, exchange=None) -> "ShardedTable":
        """This rank's shard of a resident table (for tests and small tables)."""
        rows = full.rows.view(full.n_rows, full.row_stride)[rank::world].contiguous().reshape(-1)
        return cls(rows, full.fmt, full.dim, full.head_vocab_sizes, full.head_offsets, full.layer_multipliers,
                   full.eos_token_id, world, rank, full.n_rows, full.ngram_size, full.heads_per_ngram, exchange)

    def global_ids(self, tokens, seg_start=None, t0: int = 0, n: int | None = None) -> torch.Tensor:
        """int32 [n, n_heads] global row ids (engram_hash with the table's constants)."""
        tokens = _as_i32(tokens, self.device)
        if n is None:
            n = tokens.numel() - t0
        ss = None if seg_start is None else _as_i32(seg_start, self.device)
        ids = torch.empty(n, self.n_heads, dtype=torch.int32, device=self.device)
        st = L.load().engram_hash(C.byref(self.ctable), tokens.data_ptr(), L.ptr(ss), t0, n, ids.data_ptr(),
                                  L.stream_of(self.device))
        L.check(st, "engram_hash")
        return ids

    def requests(self, ids: torch.Tensor, slots: torch.Tensor | None):
        """(send_ids [U] grouped by owner, send_counts list[W], row_index [n])."""
        lib = L.load()
        n = ids.numel()
        cap = max(2, 1 << int(np.ceil(np.log2(max(2 * n, 2)))))
        keys = torch.empty(cap, dtype=torch.int32, device=self.device)
        vals = torch.empty(cap, dtype=torch.int32, device=self.device)
        send = torch.empty(max(n, 1), dtype=torch.int32, device=self.device)
        counts = torch.empty(2 * self.world, dtype=torch.int64, device=self.device)
        rix = torch.empty(max(n, 1), dtype=torch.int32, device=self.device)
        st = lib.engram_shard_requests(ids.data_ptr(), L.ptr(slots), n, self.world, keys.data_ptr(), vals.data_ptr(),
                                       cap, send.data_ptr(), counts.data_ptr(), rix.data_ptr(),
                                       L.stream_of(self.device))
        L.check(st, "engram_shard_requests")
        send_counts = counts[: self.world].tolist()  # host sync: NCCL needs the split sizes
        return send[: sum(send_counts)], send_counts, rix[:n]

    def serve(self, recv_ids: torch.Tensor) -> torch.Tensor:
        """Owner side: the resident rows of recv_ids from this shard, uint8 [n*stride]."""
        out = torch.empty(max(recv_ids.numel(), 1) * self.stride, dtype=torch.uint8, device=self.device)
        st = L.load().engram_shard_gather(self.shard.data_ptr(), self.stride, self.n_local, recv_ids.data_ptr(),
                                          recv_ids.numel(), self.world, out.data_ptr(), L.stream_of(self.device))
        L.check(st, "engram_shard_gather")
        return out[: recv_ids.numel() * self.stride]

    def fetch(self, ids: torch.Tensor, slots: torch.Tensor | None, exchange):
        """Rows for every (position, head) of `ids` the overlay does not serve:
        (rows uint8 [U*stride] in send order, row_index [n])."""
        send_ids, send_counts, rix = self.requests(ids, slots)
        rows = exchange(self, send_ids, send_counts)
        return rows, rix

    @staticmethod
    def _key(tokens: torch.Tensor, ss: torch.Tensor | None, t0: int, n: int):
        return (tokens.data_ptr(), tokens._version, 0 if ss is None else ss.data_ptr(),
                -1 if ss is None else ss._version, int(t0), int(n))

    def enable_push_staging(self, n_tokens_max: int, group=None, max_blocks: int = 0) -> None:
        """Make prefetch() push-based and collective: every rank's tokens go to
        symmetric memory, and each owner copies the rows it holds into the
        requesters' stage buffers with NVLink stores (engram_stage_push) instead
        of each rank pulling its rows with NVLink loads.  Every rank of the
        group then calls prefetch() and forward() in the same order, with the
        same t0 and n and with or without seg_start alike; n_tokens_max bounds
        the token arrays.  A collective: every rank calls it."""
        if self.peer_ptrs is None:
            raise RuntimeError("push staging needs the peer shards (peer_ptrs)")
        self.push = PushStage(self, n_tokens_max, group, max_blocks)

    def enable_exchange_staging(self, n_tokens_max: int, exchange=None, dedup: bool = False) -> None:
        """Make prefetch() route and exchange the rows of other ranks ahead of
        the forward through `exchange`: "peer" (PeerRowExchange, the default:
        requests pushed into the owners' memory, owners gather locally,
        requesters copy with the copy engines), "nccl" (NcclRowExchange: NCCL
        all-to-alls on a process group of their own) or an exchange object
        (LocalPeerRowExchange or LocalRowExchange for emulated ranks).
        dedup: request each distinct remote row once per batch
        (engram_shard_plan, a device hash set) instead of once per (position,
        head); it needs a counting exchange, so with exchange None it selects
        "nccl".  Prefetching three batches ahead of the forward keeps both the
        host and the forward from waiting on the exchange (ExchangeStage).  A
        collective: every rank calls it."""
        if exchange is None:
            exchange = "nccl" if dedup else "peer"
        if exchange == "peer":
            exchange = PeerRowExchange(self, n_tokens_max)
        elif exchange == "nccl":
            exchange = NcclRowExchange()
        self.xstage = ExchangeStage(self, n_tokens_max, exchange, dedup)

    def prefetch(self, tokens, seg_start=None, t0: int = 0, n: int | None = None, max_blocks: int = 0,
                 stream: torch.cuda.Stream | None = None, omap: OverlayMap | None = None,
                 ready: torch.cuda.Event | None = None) -> None:
        """Copy the rows of other ranks that forward(tokens, seg_start, ..., t0, n)
        will read into this GPU's memory, on `stream` (default: the table's own
        side stream, ordered after the work already queued on the current
        stream).  The next forward() over the same int32 device tensors (same
        storage, not modified since) waits for the copy and reads those rows
        locally; any other forward reads in place as before.  omap: the overlay
        map the forward will use; the rows of the heads it serves are not
        copied, and a forward with another map reads in place.  Up to two
        prefetches wait at a time; a third drops the oldest.  max_blocks caps the
        copy's grid (0: every SM), leaving SMs to the work it overlaps.
        ready (exchange staging): an event after which tokens and seg_start
        hold their values; the staging then waits for that event only, not for
        all the work queued on the current stream, and overlaps it fully."""
        dev = self.device
        tokens = _as_i32(tokens, dev)
        if n is None:
            n = tokens.numel() - t0
        ss = None if seg_start is None else _as_i32(seg_start, dev)
        key = self._key(tokens, ss, t0, n)
        if self.xstage is not None:
            self.xstage.prefetch(key, tokens, ss, t0, n, omap, ready)
            return
        if self.peer_ptrs is None:
            raise RuntimeError("prefetch needs the peer shards (peer_ptrs) or exchange staging")
        if self.world == 1:
            return
        if self.push is not None:
            self.push.prefetch(key, tokens, ss, t0, n)
            return
        if key in self._staged:
            return
        while len(self._staged) >= 2:
            self._free.append(self._staged.popitem(last=False)[1])
        need = max(int(L.load().engram_stage_bytes(C.byref(self.ctable), n)), 16)
        L.check(min(need, 0), "engram_stage_bytes")
        slot = next((f for f in self._free if f.buf.numel() >= need), None)
        if slot is None:
            if self._free:  # grow the smallest buffer
                slot = min(self._free, key=lambda f: f.buf.numel())
                slot.buf = torch.empty(need, dtype=torch.uint8, device=dev)
            else:
                slot = _Staged(torch.empty(need, dtype=torch.uint8, device=dev))
        else:
            self._free.remove(slot)
        cur = torch.cuda.current_stream(dev)
        if stream is None:
            if self._side is None:
                self._side = torch.cuda.Stream(dev)
            stream = self._side
        stream.wait_stream(cur)
        if slot.consumed is not None:  # the previous forward over this buffer has read it
            stream.wait_event(slot.consumed)
        ov = None
        if omap is not None and omap.R:
            ov = L.EngramOverlay(None, omap.R, omap.keys.data_ptr(), omap.slots.data_ptr(), omap.capacity)
        st = L.load().engram_stage_sharded(C.byref(self.ctable), None if ov is None else C.byref(ov),
                                           tokens.data_ptr(), L.ptr(ss), t0, n, self.peer_ptrs.data_ptr(), self.world,
                                           self.rank, slot.buf.data_ptr(), int(max_blocks), stream.cuda_stream)
        L.check(st, "engram_stage_sharded")
        slot.omap = None if ov is None else omap.keys.data_ptr()
        tokens.record_stream(stream)
        if ss is not None:
            ss.record_stream(stream)
        slot.ready = torch.cuda.Event()
        slot.ready.record(stream)
        slot.consumed = None
        slot.keep = (tokens, ss)
        self._staged[key] = slot

    def forward(self, tokens, seg_start, omap: OverlayMap, rows_var, out: torch.Tensor, mode: int,
                exchange=None, slots_out=None, hit_count=None, t0: int = 0, n: int | None = None):
        """With peer_ptrs: one fused forward reading rows from their owners.
        Otherwise: hash -> overlay lookup -> row exchange -> forward over the
        received rows."""
        lib = L.load()
        dev = self.device
        tokens = _as_i32(tokens, dev)
        if n is None:
            n = tokens.numel() - t0
        ss = None if seg_start is None else _as_i32(seg_start, dev)
        stream = L.stream_of(dev)
        if self.xstage is not None:
            key = self._key(tokens, ss, t0, n)
            if not self.xstage.has(key):  # not prefetched: plan and exchange now (the host waits for the plan)
                self.xstage.prefetch(key, tokens, ss, t0, n, omap)
            b, recv, rix, ready = self.xstage.take(key, omap)
            cur = torch.cuda.current_stream(dev)
            t_wait = self.xstage._mark(cur)
            cur.wait_event(ready)
            self.xstage._span("wait", t_wait, cur)
            ov = omap.descriptor(rows_var)
            st = lib.engram_forward_exchanged(C.byref(self.ctable), C.byref(ov), tokens.data_ptr(), L.ptr(ss), t0, n,
                                              self.shard.data_ptr(), self.world, self.rank, recv.data_ptr(),
                                              rix.data_ptr(), mode, out.data_ptr(), None, L.ptr(slots_out),
                                              L.ptr(hit_count), stream)
            L.check(st, "engram_forward_exchanged")
            self.xstage.consumed(b, cur)
            return out
        if self.peer_ptrs is not None and exchange is None:
            ov = omap.descriptor(rows_var)
            key = self._key(tokens, ss, t0, n)
            if self.push is not None and self.push.has(key):
                b, buf, rix, ready = self.push.take(key)
                cur = torch.cuda.current_stream(dev)
                cur.wait_event(ready)
                desc = L.EngramTable.from_buffer_copy(self.ctable)
                desc.rows = buf.data_ptr()
                desc.n_rows = max(1, n * self.n_heads)
                st = lib.engram_forward_indirect(C.byref(desc), C.byref(ov), tokens.data_ptr(), L.ptr(ss), t0, n,
                                                 rix.data_ptr(), mode, out.data_ptr(), None, L.ptr(slots_out),
                                                 L.ptr(hit_count), stream)
                L.check(st, "engram_forward_indirect")
                self.push.consumed(b, cur)
                return out
            slot = self._staged.pop(key, None) if self._staged else None
            if slot is not None and slot.omap is not None and (not omap.R or omap.keys.data_ptr() != slot.omap):
                self._free.append(slot)  # staged without the rows of another overlay's heads: read in place
                slot = None
            if slot is not None:
                cur = torch.cuda.current_stream(dev)
                cur.wait_event(slot.ready)
                st = lib.engram_forward_staged(C.byref(self.ctable), C.byref(ov), tokens.data_ptr(), L.ptr(ss), t0,
                                               n, self.peer_ptrs.data_ptr(), self.world, self.rank,
                                               slot.buf.data_ptr(), mode, out.data_ptr(), None, L.ptr(slots_out),
                                               L.ptr(hit_count), stream)
                L.check(st, "engram_forward_staged")
                slot.consumed = torch.cuda.Event()
                slot.consumed.record(cur)
                slot.keep = None
                self._free.append(slot)
                return out
            st = lib.engram_forward_sharded(C.byref(self.ctable), C.byref(ov), tokens.data_ptr(), L.ptr(ss), t0, n,
                                            self.peer_ptrs.data_ptr(), self.world, mode, out.data_ptr(), None,
                                            L.ptr(slots_out), L.ptr(hit_count), stream)
            L.check(st, "engram_forward_sharded")
            return out
        if exchange is None:
            raise RuntimeError("this ShardedTable has neither peer shards nor a row exchange")
        ids = self.global_ids(tokens, ss, t0, n)
        ov = omap.descriptor(rows_var)
        slots = None
        if omap.R:
            slots = torch.empty_like(ids)
            st = lib.engram_overlay_lookup(C.byref(ov), ids.data_ptr(), ids.numel(), slots.data_ptr(), stream)
            L.check(st, "engram_overlay_lookup")
        rows, rix = self.fetch(ids.reshape(-1), None if slots is None else slots.reshape(-1), exchange)
        desc = L.EngramTable.from_buffer_copy(self.ctable)
        rows_buf = rows if rows.numel() else torch.zeros(16, dtype=torch.uint8, device=dev)
        desc.rows = rows_buf.data_ptr()
        desc.n_rows = max(1, rows.numel() // self.stride)
        st = lib.engram_forward_indirect(C.byref(desc), C.byref(ov), tokens.data_ptr(), L.ptr(ss), t0, n,
                                         rix.data_ptr(), mode, out.data_ptr(), None, L.ptr(slots_out),
                                         L.ptr(hit_count), stream)
        L.check(st, "engram_forward_indirect")
        self._keep = (rows_buf, rix, ids)  # alive until the stream has consumed them
        return out


class PushStage:
    """Collective, push-based staging for a row-sharded table in peer memory.

    Each rank's stage holds every row of its next forward, grouped by owner
    (engram_stage_plan), so each owner writes a requester's rows as one
    contiguous run of NVLink stores (engram_stage_push) and the forward reads
    local HBM through a row index (engram_forward_indirect).  Buffers, two sets
    (batch j uses set j % 2): in symmetric memory the tokens and segment
    starts [n_tokens_max], the plan [world * (ceil(n_tokens_max / 32) + 1)]
    and the stage [n_tokens_max * n_heads * row_stride bytes]; locally the row
    index [n_tokens_max * n_heads].  On the table's side stream, prefetch(j):
      copy this rank's tokens (and segment starts) into set b; plan the stage;
      wait until this rank's forward over set b's previous batch is done;
      barrier (4-byte NCCL all-reduce on a group of its own): every rank's
        tokens and plan of batch j are in place, every rank's stage b is free,
        and every owner's copy for batch j-1 has landed (batch j-1 is ready);
      engram_stage_push: this rank's rows of every rank's batch j go into that
        rank's stage b.
    A forward over batch j waits for the next barrier after its push: the one
    in prefetch(j+1), or one the forward issues itself if prefetch(j+1) has
    not been called.  No kernel waits on another GPU."""

    def __init__(self, table: "ShardedTable", n_tokens_max: int, group=None, max_blocks: int = 0):
        import torch.distributed as dist
        from .dist import symmetric_memory
        symm = symmetric_memory()
        group = group if group is not None else dist.group.WORLD
        if dist.get_world_size(group) != table.world or dist.get_rank(group) != table.rank:
            raise ValueError("the group's ranks must be the table's ranks")
        self.table = table
        self.dist = dist
        dev = table.device
        lib = L.load()
        self.n_max = int(n_tokens_max)
        self.max_blocks = int(max_blocks)
        stage_bytes = max(self.n_max * table.n_heads * table.stride, 16)
        plan_words = max(int(lib.engram_stage_plan_words(self.n_max, table.world)), 1)
        self.tok, self.seg, self.plan, self.stage, self.rix, self._handles, self.ptrs = [], [], [], [], [], [], []
        for _ in range(2):
            bufs = (symm.empty(max(self.n_max, 1), dtype=torch.int32, device=dev),
                    symm.empty(max(self.n_max, 1), dtype=torch.int32, device=dev),
                    symm.empty(plan_words, dtype=torch.int32, device=dev),
                    symm.empty(stage_bytes, dtype=torch.uint8, device=dev))
            hs = [symm.rendezvous(x, group) for x in bufs]
            for lst, x in zip((self.tok, self.seg, self.plan, self.stage), bufs):
                lst.append(x)
            self._handles.append(hs)
            # per set: token, segment, plan and stage pointers of every rank, valid in this process
            self.ptrs.append(tuple(torch.tensor(list(h.buffer_ptrs), dtype=torch.int64, device=dev) for h in hs))
            self.rix.append(torch.empty(max(self.n_max * table.n_heads, 1), dtype=torch.int32, device=dev))
        # the barrier gets a communicator of its own, so it never queues behind the step's collectives
        self.group = dist.new_group(ranks=list(range(table.world)))
        self.side = torch.cuda.Stream(dev)
        self.flag = torch.zeros(1, dtype=torch.int32, device=dev)
        self.j = 0  # batches prefetched so far
        self.keys = {}  # key -> set index, pushed and not yet read
        self.ready = [None, None]  # event after the barrier that completed set b's pushes
        self.done = [None, None]  # event after the forward that read set b
        self.unbarriered = None  # set whose push no barrier has followed yet

    def _barrier(self) -> None:
        with torch.cuda.stream(self.side):
            self.dist.all_reduce(self.flag, group=self.group)
        if self.unbarriered is not None:
            ev = torch.cuda.Event()
            ev.record(self.side)
            self.ready[self.unbarriered] = ev
            self.unbarriered = None

    def prefetch(self, key, tokens: torch.Tensor, ss: torch.Tensor | None, t0: int, n: int) -> None:
        t = self.table
        if tokens.numel() > self.n_max or t0 + n > self.n_max:
            raise ValueError(f"{tokens.numel()} tokens (t0 + n = {t0 + n}) exceed n_tokens_max {self.n_max}")
        b = self.j % 2
        self.j += 1
        for k in [k for k, v in self.keys.items() if v == b]:  # a batch pushed two prefetches ago, never read
            del self.keys[k]
        lib = L.load()
        cur = torch.cuda.current_stream(t.device)
        self.side.wait_stream(cur)
        with torch.cuda.stream(self.side):
            self.tok[b][: tokens.numel()].copy_(tokens)
            if ss is not None:
                self.seg[b][: ss.numel()].copy_(ss)
        tokens.record_stream(self.side)
        if ss is not None:
            ss.record_stream(self.side)
        st = lib.engram_stage_plan(C.byref(t.ctable), self.tok[b].data_ptr(),
                                   None if ss is None else self.seg[b].data_ptr(), t0, n, t.world,
                                   self.plan[b].data_ptr(), self.rix[b].data_ptr(), self.side.cuda_stream)
        L.check(st, "engram_stage_plan")
        if self.done[b] is not None:
            self.side.wait_event(self.done[b])
        self._barrier()
        tp, sp, pp, stp = self.ptrs[b]
        st = lib.engram_stage_push(C.byref(t.ctable), tp.data_ptr(), None if ss is None else sp.data_ptr(),
                                   pp.data_ptr(), t0, n, stp.data_ptr(), t.world, t.rank, self.max_blocks,
                                   self.side.cuda_stream)
        L.check(st, "engram_stage_push")
        self.ready[b] = None
        self.unbarriered = b
        self.keys[key] = b

    def has(self, key) -> bool:
        return key in self.keys

    def take(self, key):
        """(set index, this rank's stage, its row index, the event after which
        every owner's rows are in the stage)."""
        b = self.keys.pop(key)
        if self.ready[b] is None:  # no prefetch has followed this batch's push: close it now
            self._barrier()
        return b, self.stage[b], self.rix[b], self.ready[b]

    def consumed(self, b: int, stream: torch.cuda.Stream) -> None:
        """The forward reading set b is queued on `stream`: the next push into b waits for it."""
        ev = torch.cuda.Event()
        ev.record(stream)
        self.done[b] = ev

    def join(self, stream: torch.cuda.Stream) -> None:
        """`stream` waits for the staging in flight, the barrier that completes it included."""
        if self.unbarriered is not None:
            self._barrier()
        stream.wait_stream(self.side)


class ExchangeStage:
    """Row-sharded reads through a row exchange, pipelined so that neither the
    host nor the forward waits for it (ShardedTable.enable_exchange_staging).

    A batch passes three stages, one per prefetch() call, so a caller that
    prefetches three batches ahead of its forwards has, at step k: batch k+3
    routed, batch k+2 served, batch k+1 fetched, batch k read by the forward.

    With a pushing exchange (PeerRowExchange, LocalPeerRowExchange; the
    default), one prefetch() call queues on the caller's stream:
      serve: the owners' gather of the batch routed one call earlier
        (engram_shard_serve_pushed, local reads and writes only);
      route: engram_shard_route_push for the new batch, which stores each
        remote (position, head) pair's id straight into its owner's request
        buffer and its counts into the owner's count array, and a copy of this
        rank's counts to pinned host memory;
      barrier: a 4-byte all-reduce.  Once it completes, every rank's route of
        this call is visible to its owners (served next call) and every
        owner's gather of this call is done (fetched next call);
    and on the side stream, at the end of the next prefetch() call (after
    its barrier, so the copies overlap the forward that follows rather than
    the gathers and the route, which move more bytes per unit time):
      fetch: the batch's rows, one copy-engine transfer per owner from the
        owner's send buffer (the host reads this rank's counts, copied two
        calls earlier, so it does not wait).  Queued behind the forward
        instead, the copies slowed the backward more than they slow the
        forward here (N = 2: backward 0.157 -> 0.223 ms).
    No collective runs on the side stream: it carries only copy-engine
    transfers, so nothing there competes with the forward for SMs.

    With a counting exchange (NcclRowExchange, LocalRowExchange):
      route (current stream): engram_shard_route (engram_shard_plan with
        dedup: each distinct row once), the ids grouped by owner in a local
        send_ids; then, on the side stream, every rank's counts are
        all-gathered (exchange.gather_counts) and copied to the host;
      serve: nothing;
      fetch (side stream): exchange.rows moves ids out and rows back.

    forward(X) runs the stages X has not passed yet (the host then waits),
    makes the current stream wait for X's rows and runs
    engram_forward_exchanged.  Every rank calls prefetch and forward in the
    same order with the same t0 and n (the collectives and the buffer sets
    follow that order).  Four buffer sets: a fifth batch prefetched before the
    oldest is read drops the oldest."""

    SETS = 4

    def __init__(self, table: "ShardedTable", n_tokens_max: int, exchange, dedup: bool = False):
        self.table, self.exchange = table, exchange
        self.dedup = bool(dedup)  # engram_shard_plan (distinct rows) or engram_shard_route (one row per pair)
        self.push = bool(getattr(exchange, "pushes", False))
        if self.push and self.dedup:
            raise ValueError("dedup needs a counting exchange (\"nccl\" or LocalRowExchange)")
        dev = table.device
        self.n_max = int(n_tokens_max)
        entries = max(self.n_max * table.n_heads, 1)
        self.cap = max(2, 1 << int(np.ceil(np.log2(2 * entries))))
        self.set_keys = torch.empty(self.cap, dtype=torch.int32, device=dev)
        self.set_vals = torch.empty(self.cap if self.dedup else 1, dtype=torch.int32, device=dev)
        W = table.world
        alloc = getattr(exchange, "alloc_ids", None)
        if self.push:  # the route stores the ids in the owners' request buffers
            self.send_ids = [None] * self.SETS
        else:
            self.send_ids = [alloc(b, entries) if alloc is not None
                             else torch.empty(entries, dtype=torch.int32, device=dev) for b in range(self.SETS)]
        self.rix = [torch.empty(entries, dtype=torch.int32, device=dev) for _ in range(self.SETS)]
        self.counts = [torch.zeros(2 * W, dtype=torch.int64, device=dev) for _ in range(self.SETS)]
        self.counts_host = [torch.zeros(W, W, dtype=torch.int64).pin_memory() for _ in range(self.SETS)]
        self.allc = [None] * self.SETS        # every rank's counts, on the device
        self.ev_counts = [None] * self.SETS   # side: counts gathered and copied to the host
        self.ev_barrier = [None] * self.SETS  # every owner's gather of the batch is done
        self.ev_ready = [None] * self.SETS    # side: the batch's rows are in its receive buffer
        self.recv = [None] * self.SETS
        self.state = [None] * self.SETS       # None | "routed" | "served" | "fetched"
        self.key = [None] * self.SETS
        self.omap_keys = [None] * self.SETS
        self.seq = [0] * self.SETS
        self.n_seq = 0
        self.side = torch.cuda.Stream(dev)
        self._empty = torch.zeros(16, dtype=torch.uint8, device=dev)
        self.timing = None  # a dict of lists of (start, end) CUDA events per phase, when set (see phase_ms)

    def has(self, key) -> bool:
        return key in self.key

    def _mark(self, stream):
        if self.timing is None:
            return None
        e = torch.cuda.Event(enable_timing=True)
        e.record(stream)
        return e

    def _span(self, name, e0, stream):
        if e0 is not None:
            self.timing.setdefault(name, []).append((e0, self._mark(stream)))

    def phase_ms(self) -> dict:
        """Median ms per batch of each timed phase (after a synchronize): route,
        serve and barrier on the caller's stream, fetch on the side stream,
        wait = how long the forward's stream waited for its rows."""
        out = {}
        for k, v in (self.timing or {}).items():
            if v:
                ms = sorted(a.elapsed_time(b) for a, b in v)
                out[k] = ms[len(ms) // 2]
        return out

    def _oldest(self, state):
        return sorted((k for k in range(self.SETS) if self.state[k] == state), key=lambda k: self.seq[k])

    def prefetch(self, key, tokens: torch.Tensor, ss: torch.Tensor | None, t0: int, n: int, omap,
                 ready: torch.cuda.Event | None = None) -> None:
        t = self.table
        if key in self.key:
            return
        if n > self.n_max:
            raise ValueError(f"{n} positions exceed n_tokens_max {self.n_max}")
        cur = torch.cuda.current_stream(t.device)
        fetch_now = self._oldest("served")  # the next forward waits for the oldest of them
        if not self.push:
            for b in fetch_now:
                self._fetch(b)
        served = self._oldest("routed")
        for b in served:
            self._serve(b, cur)
        free = [b for b in range(self.SETS) if self.state[b] is None]
        if not free:  # drop the oldest waiting batch (every rank drops the same one)
            b = min(range(self.SETS), key=lambda k: self.seq[k])
            self.state[b] = self.key[b] = None
            free = [b]
        b = free[0]
        if ready is not None:
            cur.wait_event(ready)
        ov = None
        if omap is not None and omap.R:
            ov = L.EngramOverlay(None, omap.R, omap.keys.data_ptr(), omap.slots.data_ptr(), omap.capacity)
        if self.push:
            if self.ev_ready[b] is not None:  # the set's last copies are done before its owners refill it
                cur.wait_event(self.ev_ready[b])
            t_route = self._mark(cur)
            self.exchange.route(t, b, ov, tokens, ss, t0, n, self.counts[b], self.rix[b], cur)
            self.counts_host[b][0].copy_(self.counts[b][: t.world], non_blocking=True)
            self._span("route", t_route, cur)
            self.ev_counts[b] = torch.cuda.Event()
            self.ev_counts[b].record(cur)
            self.allc[b] = None
            t_bar = self._mark(cur)
            self.exchange.barrier()
            self._span("barrier", t_bar, cur)
            done = torch.cuda.Event()
            done.record(cur)
            for s_ in served:
                self.ev_barrier[s_] = done
            for s_ in fetch_now:  # behind this call's gathers and route, so the copies overlap the forward
                self._fetch(s_)
            self._routed(b, key, ov, omap)
            return
        t_route = self._mark(cur)
        lib = L.load()
        if self.dedup:
            st = lib.engram_shard_plan(C.byref(t.ctable), None if ov is None else C.byref(ov), tokens.data_ptr(),
                                       L.ptr(ss), t0, n, t.world, t.rank, self.set_keys.data_ptr(),
                                       self.set_vals.data_ptr(), self.cap, self.send_ids[b].data_ptr(),
                                       self.counts[b].data_ptr(), self.rix[b].data_ptr(), cur.cuda_stream)
            L.check(st, "engram_shard_plan")
        else:
            st = lib.engram_shard_route(C.byref(t.ctable), None if ov is None else C.byref(ov), tokens.data_ptr(),
                                        L.ptr(ss), t0, n, t.world, t.rank, self.set_keys.data_ptr(), self.cap,
                                        self.send_ids[b].data_ptr(), self.counts[b].data_ptr(), self.rix[b].data_ptr(),
                                        cur.cuda_stream)
            L.check(st, "engram_shard_route")
        self._span("route", t_route, cur)
        routed = torch.cuda.Event()
        routed.record(cur)
        self.side.wait_event(routed)
        with torch.cuda.stream(self.side):
            allc = self.exchange.gather_counts(t, self.counts[b][: t.world])
            self.counts_host[b].copy_(allc.reshape(t.world, t.world), non_blocking=True)
        allc.record_stream(cur)
        self.allc[b] = allc
        self.ev_counts[b] = torch.cuda.Event()
        self.ev_counts[b].record(self.side)
        self._routed(b, key, ov, omap)

    def _routed(self, b: int, key, ov, omap) -> None:
        self.recv[b] = None
        self.state[b], self.key[b] = "routed", key
        self.omap_keys[b] = None if ov is None else omap.keys.data_ptr()
        self.n_seq += 1
        self.seq[b] = self.n_seq

    def _serve(self, b: int, cur: torch.cuda.Stream) -> None:
        if self.push:  # this owner's gather; the barrier after it comes with the call's route (or take)
            t0 = self._mark(cur)
            self.exchange.serve(self.table, b)
            self._span("serve", t0, cur)
            self.ev_barrier[b] = None
        else:
            self.ev_barrier[b] = self.ev_counts[b]
        self.state[b] = "served"

    def _fetch(self, b: int) -> None:
        t = self.table
        self.ev_counts[b].synchronize()
        m = self.counts_host[b]
        self.side.wait_event(self.ev_barrier[b])
        t0 = self._mark(self.side)
        with torch.cuda.stream(self.side):
            if self.push:
                rows = self.exchange.fetch(t, b, [int(x) for x in m[0, : t.world].tolist()])
            else:
                send = [int(x) for x in m[t.rank].tolist()]
                recv = [int(x) for x in m[:, t.rank].tolist()]
                rows = self.exchange.rows(t, self.send_ids[b][:sum(send)], send, recv)
        self._span("fetch", t0, self.side)
        self.recv[b] = rows if rows.numel() else self._empty
        self.ev_ready[b] = torch.cuda.Event()
        self.ev_ready[b].record(self.side)
        self.state[b] = "fetched"

    def take(self, key, omap):
        """(set, receive buffer, row_index, ready event) of the prefetched batch `key`."""
        b = self.key.index(key)
        want = None if omap is None or not omap.R else omap.keys.data_ptr()
        if want != self.omap_keys[b]:
            raise ValueError("the batch was prefetched with another overlay map; prefetch it again with this one")
        cur = torch.cuda.current_stream(self.table.device)
        if self.state[b] == "routed":  # its route's barrier came with the call that routed it
            self._serve(b, cur)
            if self.push:
                self.exchange.barrier()
                self.ev_barrier[b] = torch.cuda.Event()
                self.ev_barrier[b].record(cur)
        if self.state[b] == "served":
            self._fetch(b)
        self.key[b] = None
        self.recv[b].record_stream(cur)  # read by the forward there
        return b, self.recv[b], self.rix[b], self.ev_ready[b]

    def consumed(self, b: int, stream: torch.cuda.Stream) -> None:
        """The forward over set b is queued on `stream` (the set's next route
        runs on the caller's stream after it)."""
        self.state[b] = None


class NcclRowExchange:
    """The collectives of ExchangeStage over torch.distributed, on a process
    group of their own (NCCL between GPUs, gloo on CPU for tests) so they run
    beside the step's other collectives instead of queueing behind them.
    A collective to construct: every rank of `group` calls it."""

    def __init__(self, group=None):
        import torch.distributed as dist
        self.dist = dist
        base = group if group is not None else dist.group.WORLD
        self.group = dist.new_group(ranks=dist.get_process_group_ranks(base))

    def gather_counts(self, table, counts: torch.Tensor) -> torch.Tensor:
        """[W*W] int64: entry r*W + o = the rows rank r requests from owner o."""
        W = table.world
        out = torch.empty(W * W, dtype=torch.int64, device=counts.device)
        self.dist.all_gather_into_tensor(out, counts.contiguous(), group=self.group)
        return out

    def rows(self, table, send_ids: torch.Tensor, send_counts, recv_counts) -> torch.Tensor:
        """The rows of send_ids (grouped by owner, send_counts per owner) from
        their owners, in send order: ids out (all-to-all), each owner gathers
        the rows asked of it (ShardedTable.serve), rows back (all-to-all)."""
        dev = send_ids.device
        recv_ids = torch.empty(max(sum(recv_counts), 1), dtype=torch.int32, device=dev)[: sum(recv_counts)]
        self.dist.all_to_all_single(recv_ids, send_ids, recv_counts, send_counts, group=self.group)
        served = table.serve(recv_ids)
        stride = table.stride
        rows = torch.empty(max(sum(send_counts), 1) * stride, dtype=torch.uint8, device=dev)[: sum(send_counts) * stride]
        self.dist.all_to_all_single(rows, served, [c * stride for c in send_counts],
                                    [c * stride for c in recv_counts], group=self.group)
        return rows


class _PushExchange:
    """The buffers and calls of a pushing exchange, per batch set b: this
    owner's request buffer ids[b] (int32 [world, region]), count array
    cnts[b] (int64 [world]) and send buffer rows[b] ([world, region] rows),
    with device tables of every rank's request buffer and count array
    (id_ptrs[b], cnt_ptrs[b]).  Subclasses say where the buffers live, how the
    owners' send buffers are reached and what the barrier is."""

    pushes = True

    def _setup(self, table: "ShardedTable", n_tokens_max: int, sets: int) -> None:
        W = table.world
        self.world, self.rank, self.stride, self.sets = W, table.rank, table.stride, sets
        self.region = max(int(n_tokens_max) * table.n_heads, 1)  # a batch's pairs: the most one owner can get
        if W * self.region > 2**31 - 1:
            raise ValueError(f"{W} ranks x {self.region} pairs per batch exceed the int32 row tags")
        self.ids, self.cnts, self.rows, self.id_ptrs, self.cnt_ptrs = [], [], [], [], []

    def route(self, table, b: int, ov, tokens: torch.Tensor, ss, t0: int, n: int, counts: torch.Tensor,
              row_index: torch.Tensor, stream: torch.cuda.Stream) -> None:
        """engram_shard_route_push for set b on `stream`."""
        st = L.load().engram_shard_route_push(C.byref(table.ctable), None if ov is None else C.byref(ov),
                                              tokens.data_ptr(), L.ptr(ss), t0, n, self.world, self.rank,
                                              self.id_ptrs[b].data_ptr(), self.cnt_ptrs[b].data_ptr(), self.region,
                                              counts.data_ptr(), row_index.data_ptr(), stream.cuda_stream)
        L.check(st, "engram_shard_route_push")

    def serve(self, table, b: int) -> None:
        """This owner's gather for set b, on the current stream."""
        st = L.load().engram_shard_serve_pushed(table.shard.data_ptr(), table.stride, table.n_local, self.world,
                                                self.rank, self.ids[b].data_ptr(), self.cnts[b].data_ptr(),
                                                self.region, self.rows[b].data_ptr(), L.stream_of(table.device))
        L.check(st, "engram_shard_serve_pushed")

    def _send_rows(self, b: int, o: int) -> torch.Tensor:
        raise NotImplementedError

    def _before_fetch(self, b: int) -> None:
        pass

    def fetch(self, table, b: int, own) -> torch.Tensor:
        """This rank's rows of set b (own[o] = the rows it asked of owner o), in
        ascending owner order: one copy-engine transfer per owner from the
        start of this rank's region of the owner's send buffer."""
        W, me, stride, region = self.world, self.rank, self.stride, self.region
        total = sum(own)
        out = torch.empty(max(total, 1) * stride, dtype=torch.uint8, device=table.device)
        self._before_fetch(b)
        off = 0
        for o in range(W):
            cnt = own[o]
            if o == me or cnt == 0:
                continue
            if cnt > region:
                raise RuntimeError(f"{cnt} rows asked of owner {o}, its region holds {region}")
            src = self._send_rows(b, o)[me * region * stride:(me * region + cnt) * stride]
            out[off * stride:(off + cnt) * stride].copy_(src, non_blocking=True)
            off += cnt
        return out[: total * stride]


class PeerRowExchange(_PushExchange):
    """ExchangeStage's exchange between GPUs over peer memory: requests pushed
    into the owners' memory by the route, owners gather locally, requesters
    copy their rows with the copy engines.

    Every buffer lives in torch symmetric memory (no multicast object), so
    each rank's request buffers and count arrays are written by the others
    (plain stores from engram_shard_route_push) and its send buffers are read
    by the others' copy engines (torch copy_ from a peer view, one
    cudaMemcpyAsync per owner: NVLink, no SMs).  The barrier is a 4-byte
    all-reduce on a process group of the exchange's own.  A collective to
    construct: every rank of `group` calls it."""

    def __init__(self, table: "ShardedTable", n_tokens_max: int, group=None, sets: int = 4):
        import torch.distributed as dist
        from .dist import symmetric_memory
        symm = symmetric_memory()
        self.dist = dist
        base = group if group is not None else dist.group.WORLD
        self.group = dist.new_group(ranks=dist.get_process_group_ranks(base))
        self._setup(table, n_tokens_max, sets)
        W, dev = self.world, table.device
        self.row_handles, self._keep = [], []
        for _ in range(sets):
            ids = symm.empty(W * self.region, dtype=torch.int32, device=dev)
            hi = symm.rendezvous(ids, self.group)
            cnts = symm.empty(max(W, 2), dtype=torch.int64, device=dev)
            hc = symm.rendezvous(cnts, self.group)
            rows = symm.empty(W * self.region * self.stride, dtype=torch.uint8, device=dev)
            hr = symm.rendezvous(rows, self.group)
            self.ids.append(ids)
            self.cnts.append(cnts)
            self.rows.append(rows)
            self.id_ptrs.append(torch.tensor(list(hi.buffer_ptrs), dtype=torch.int64, device=dev))
            self.cnt_ptrs.append(torch.tensor(list(hc.buffer_ptrs), dtype=torch.int64, device=dev))
            self.row_handles.append(hr)
            self._keep += [hi, hc]
        self.flag = torch.zeros(1, dtype=torch.int32, device=dev)
        self._views = {}

    def _send_rows(self, b: int, o: int) -> torch.Tensor:
        """Owner o's send buffer of set b, mapped into this process (cached)."""
        key = (b, o)
        if key not in self._views:
            self._views[key] = self.row_handles[b].get_buffer(o, (self.rows[b].numel(),), torch.uint8)
        return self._views[key]

    def barrier(self) -> None:
        """A 4-byte all-reduce on the current stream: once it completes, the
        work every rank queued before it is done."""
        self.dist.all_reduce(self.flag, group=self.group)


class LocalPeerRowExchange(_PushExchange):
    """The pushing exchange among W ranks emulated in one process on one GPU
    (tests): one object per emulated rank, made by `LocalPeerRowExchange.
    for_shards`, buffers in plain device memory.  The emulated ranks' calls
    must interleave as real ranks' would: every rank's prefetch of a step
    before any rank's next prefetch.  Each owner's gather records an event,
    and a fetch waits for the gathers of every owner (the barrier's part)."""

    def __init__(self, table: "ShardedTable", n_tokens_max: int, sets: int = 4):
        self._setup(table, n_tokens_max, sets)
        W, dev = self.world, table.device
        for _ in range(sets):
            self.ids.append(torch.empty(W * self.region, dtype=torch.int32, device=dev))
            self.cnts.append(torch.zeros(max(W, 2), dtype=torch.int64, device=dev))
            self.rows.append(torch.empty(W * self.region * self.stride, dtype=torch.uint8, device=dev))
        self.served = [None] * sets
        self.peers = None

    @classmethod
    def for_shards(cls, shards, n_tokens_max: int, sets: int = 4) -> list:
        exs = [cls(sh, n_tokens_max, sets) for sh in shards]
        for x in exs:
            x.peers = exs
            for b in range(sets):
                x.id_ptrs.append(torch.tensor([p.ids[b].data_ptr() for p in exs], dtype=torch.int64,
                                              device=shards[0].device))
                x.cnt_ptrs.append(torch.tensor([p.cnts[b].data_ptr() for p in exs], dtype=torch.int64,
                                               device=shards[0].device))
        return exs

    def serve(self, table, b: int) -> None:
        super().serve(table, b)
        self.served[b] = torch.cuda.Event()
        self.served[b].record(torch.cuda.current_stream(table.device))

    def barrier(self) -> None:
        pass

    def _before_fetch(self, b: int) -> None:
        cur = torch.cuda.current_stream(self.rows[b].device)
        for p in self.peers:
            if p is not self and p.served[b] is not None:
                cur.wait_event(p.served[b])

    def _send_rows(self, b: int, o: int) -> torch.Tensor:
        return self.peers[o].rows[b]


class LocalRowExchange:
    """ExchangeStage's exchange among shards held by one process (emulated
    ranks, for tests): every owner serves from its own ShardedTable."""

    def __init__(self, shards):
        self.shards = shards

    def gather_counts(self, table, counts: torch.Tensor) -> torch.Tensor:
        W = table.world
        out = torch.zeros(W, W, dtype=torch.int64, device=counts.device)
        out[table.rank] = counts
        return out.reshape(-1)

    def rows(self, table, send_ids: torch.Tensor, send_counts, recv_counts) -> torch.Tensor:
        parts, off = [], 0
        for owner, c in enumerate(send_counts):
            if c:
                parts.append(self.shards[owner].serve(send_ids[off:off + c]))
            off += c
        return torch.cat(parts) if parts else torch.empty(0, dtype=torch.uint8, device=send_ids.device)


class _Staged:
    """A prefetch buffer: rows of other ranks for one forward call."""
    __slots__ = ("buf", "ready", "consumed", "keep", "omap")

    def __init__(self, buf: torch.Tensor):
        self.buf = buf
        self.omap = None  # keys pointer of the overlay map whose heads were not copied
        self.ready = None  # event: the copy has landed
        self.consumed = None  # event: the forward that read it is done
        self.keep = None  # inputs of the copy, alive until the forward is issued


def nccl_exchange(group=None):
    """Exchange over torch.distributed (NCCL): ids to owners, rows back."""
    import torch.distributed as dist

    def run(shard: ShardedTable, send_ids: torch.Tensor, send_counts):
        dev = shard.device
        W = shard.world
        sc = torch.tensor(send_counts, dtype=torch.int64, device=dev)
        rc = torch.empty(W, dtype=torch.int64, device=dev)
        dist.all_to_all_single(rc, sc, group=group)
        recv_counts = rc.tolist()
        recv_ids = torch.empty(max(sum(recv_counts), 1), dtype=torch.int32, device=dev)[: sum(recv_counts)]
        dist.all_to_all_single(recv_ids, send_ids, recv_counts, send_counts, group=group)
        served = shard.serve(recv_ids)
        rows = torch.empty(max(sum(send_counts), 1) * shard.stride, dtype=torch.uint8,
                           device=dev)[: sum(send_counts) * shard.stride]
        dist.all_to_all_single(rows, served, [c * shard.stride for c in send_counts],
                               [c * shard.stride for c in recv_counts], group=group)
        return rows

    return run


def local_exchange(shards: list[ShardedTable]):
    """Exchange among W shards held by one process (emulated ranks, for tests)."""

    def run(shard: ShardedTable, send_ids: torch.Tensor, send_counts):
        parts, off = [], 0
        for owner, c in enumerate(send_counts):
            parts.append(shards[owner].serve(send_ids[off:off + c]))
            off += c
        return torch.cat(parts) if parts else torch.empty(0, dtype=torch.uint8, device=shard.device)

    return run


def peer_shard_buffer(n_rows: int, fmt: int, dim: int, device, group=None):
    """(this rank's shard buffer, ptrs): a uint8 buffer for ceil(n_rows / W)
    resident rows in torch symmetric memory, and the int64 device tensor of
    every rank's buffer address in this process (for ShardedTable's
    peer_ptrs).  A collective: every rank of the group calls it."""
    import torch.distributed as dist
    from .dist import symmetric_memory
    symm = symmetric_memory()
    group = group if group is not None else dist.group.WORLD
    world = dist.get_world_size(group)
    stride = int(L.load().engram_row_stride(fmt, dim))
    rows_max = -(-int(n_rows) // world)
    buf = symm.empty(max(rows_max * stride, 16), dtype=torch.uint8, device=device)
    h = symm.rendezvous(buf, group)
    ptrs = torch.tensor(list(h.buffer_ptrs), dtype=torch.int64, device=device)
    return buf, ptrs, h
