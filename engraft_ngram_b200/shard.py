"""Row-sharded resident table across W GPUs: owner(g) = g mod W, local index g / W.

Each rank holds 1/W of the table.  Two ways to read it:
- peer memory (peer_ptrs set): every rank's shard lives in torch symmetric
  memory, so the forward kernels copy each row straight from its owner over
  NVLink (engram_forward_sharded); nothing runs before the forward;
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
        if self.peer_ptrs is not None and exchange is None:
            ov = omap.descriptor(rows_var)
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
    import torch.distributed._symmetric_memory as symm
    group = group if group is not None else dist.group.WORLD
    world = dist.get_world_size(group)
    stride = int(L.load().engram_row_stride(fmt, dim))
    rows_max = -(-int(n_rows) // world)
    buf = symm.empty(max(rows_max * stride, 16), dtype=torch.uint8, device=device)
    h = symm.rendezvous(buf, group)
    ptrs = torch.tensor(list(h.buffer_ptrs), dtype=torch.int64, device=device)
    return buf, ptrs, h
