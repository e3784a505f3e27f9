"""Differentiable overlay gather: the drop-in for the reference's OverlayEmb.

`OverlayEmb` here has the constructor, `build()` signature, result and
attributes of engraft.replica.seq.OverlayEmb (engraft/replica/seq.py:237-444):
for positions start..n_positions-1 it returns the PLE embedding
[n_positions-start, n_heads*dim] on rows_var's device, equal to the true table
rows except where a row's global id is in row_map, where it is
rows_var[row_map[id]] -- differentiable in rows_var.  The whole build is one
fused CUDA launch (hash -> overlay probe -> gather/dequant -> emit) over the
resident table; its backward is the deterministic row-gradient kernel.

`engram_residual_add` is the builder-defined PAIRSUM mode: the bigram and
trigram rows of each of the 8 groups summed and added into a bf16 residual
stream, in place, differentiable in rows_var (and pass-through in the residual).
"""
from __future__ import annotations

import ctypes as C
import dataclasses

import numpy as np
import torch

from . import _lib as L
from .table import DeviceTable, _as_i32


class OverlayMap:
    """Device map global row id -> overlay slot (engram_overlay_map_build) for
    the keys of a reference row_map ({global_id: index}, indices 0..R-1)."""

    def __init__(self, ids: torch.Tensor, device):
        device = torch.device(device)
        ids = _as_i32(ids, device).reshape(-1)
        self.R = int(ids.numel())
        self.ids = ids
        self.peer = None  # a PeerRows exchange the autograd backward hands row gradients to (PeerRows.attach)
        self.capacity = 0 if self.R == 0 else max(2, 1 << int(np.ceil(np.log2(2 * self.R))))
        self.keys = torch.empty(max(self.capacity, 1), dtype=torch.int32, device=device)
        self.slots = torch.empty(max(self.capacity, 1), dtype=torch.int32, device=device)
        if self.R:
            st = L.load().engram_overlay_map_build(ids.data_ptr(), self.R, self.keys.data_ptr(),
                                                   self.slots.data_ptr(), self.capacity, L.stream_of(device))
            L.check(st, "engram_overlay_map_build")

    @classmethod
    def from_row_map(cls, row_map: dict, device) -> "OverlayMap":
        if any(isinstance(k, tuple) for k in row_map):
            raise NotImplementedError(
                "long (token-window, head) keys in row_map are not supported by the CUDA path "
                "(engraft/replica/seq.py:222-234 has no public producer of them)")
        R = len(row_map)
        ids = np.full(R, -1, dtype=np.int64)
        for g, i in row_map.items():
            if not (0 <= int(i) < R):
                raise ValueError(f"row_map index {i} outside [0, {R})")
            ids[int(i)] = int(g)
        if (ids < 0).any():
            raise ValueError("row_map indices must be a permutation of 0..R-1 and ids >= 0")
        if len(np.unique(ids)) != R:
            raise ValueError("row_map holds duplicate global ids")
        if R and ids.max() > 2**31 - 1:
            raise ValueError("global row id does not fit int32")
        return cls(torch.from_numpy(ids.astype(np.int32)), device)

    def descriptor(self, rows_var: torch.Tensor) -> L.EngramOverlay:
        if self.R and (rows_var.shape[0] != self.R):
            raise ValueError(f"rows_var has {rows_var.shape[0]} rows, row_map {self.R}")
        return L.EngramOverlay(rows_var.data_ptr() if self.R else None, self.R,
                               self.keys.data_ptr() if self.R else None,
                               self.slots.data_ptr() if self.R else None, self.capacity)


def seg_starts_from_segment_ids(segment_ids) -> np.ndarray:
    """seg_start[i] = first index holding segment_ids[i]'s value: the rule of
    OverlayEmb.__post_init__ (engraft/replica/seq.py:317-335); exact also for
    non-contiguous ids."""
    seg = np.asarray(segment_ids.detach().cpu() if isinstance(segment_ids, torch.Tensor) else segment_ids)
    if seg.size == 0:
        return np.zeros(0, dtype=np.int32)
    _, first, inv = np.unique(seg, return_index=True, return_inverse=True)
    return first[inv].astype(np.int32)


def _check_rows_var(rows_var: torch.Tensor, dim: int) -> None:
    if not rows_var.is_cuda:
        raise RuntimeError("the CUDA Engram path needs rows_var on a CUDA device")
    if rows_var.dtype != torch.float32:
        raise ValueError(f"rows_var must be float32, got {rows_var.dtype}")
    if rows_var.dim() != 2 or rows_var.shape[1] != dim:
        raise ValueError(f"rows_var must be [R, {dim}], got {tuple(rows_var.shape)}")


def _emit(dtable, omap: OverlayMap, rv: torch.Tensor, tokens, seg_start, t0: int, n: int, mode: int,
          out: torch.Tensor, slots, hit_count) -> None:
    """One forward launch into `out`: engram_forward on a resident table, or the
    row exchange plus engram_forward_indirect on a row-sharded table."""
    if getattr(dtable, "is_sharded", False):
        if dtable.exchange is None and dtable.peer_ptrs is None and dtable.xstage is None:
            raise RuntimeError("this ShardedTable has no way to reach other ranks' rows: set .exchange, give it "
                               "peer shards or enable exchange staging")
        dtable.forward(tokens, seg_start, omap, rv, out, mode, dtable.exchange, slots_out=slots,
                       hit_count=hit_count, t0=t0, n=n)
        return
    ov = omap.descriptor(rv)
    st = L.load().engram_forward(C.byref(dtable.ctable), C.byref(ov), tokens.data_ptr(), L.ptr(seg_start), t0, n,
                                 mode, out.data_ptr(), None, L.ptr(slots), L.ptr(hit_count),
                                 L.stream_of(dtable.device))
    L.check(st, "engram_forward")


class _ConcatFn(torch.autograd.Function):
    """emb = gather(table, overlay=rows_var) in CONCAT mode; backward = row gradients."""

    @staticmethod
    def forward(ctx, rows_var, dtable: DeviceTable, omap: OverlayMap, tokens, seg_start, t0: int, n: int,
                hit_count):
        dev = dtable.device
        nh, dim = dtable.n_heads, dtable.dim
        rv = rows_var.detach().contiguous()
        out = torch.empty(n, nh * dim, dtype=torch.float32, device=dev)
        need_grad = rows_var.requires_grad and omap.R > 0
        slots = torch.empty(n, nh, dtype=torch.int32, device=dev) if need_grad else None
        _emit(dtable, omap, rv, tokens, seg_start, t0, n, L.MODE_CONCAT_F32, out, slots, hit_count)
        ctx.meta = (nh, dtable.heads_per_ngram, dim, omap.R, n)
        ctx.peer = _peer_of(omap, rows_var)
        ctx.save_for_backward(slots if slots is not None else torch.empty(0, dtype=torch.int32, device=dev))
        return out

    @staticmethod
    def backward(ctx, grad_out):
        (slots,) = ctx.saved_tensors
        nh, hpn, dim, R, n = ctx.meta
        if not ctx.needs_input_grad[0] or R == 0 or slots.numel() == 0:
            return (None,) * 8
        grad = grad_out.contiguous().to(torch.float32)
        if ctx.peer is not None:  # row gradients stored into their owners' receive buffers; no .grad
            ctx.peer.backward(slots, grad, nh, hpn, L.MODE_CONCAT_F32)
            return (None,) * 8
        grad_rows = row_gradients(slots, grad, nh, hpn, dim, R, L.MODE_CONCAT_F32)
        return (grad_rows,) + (None,) * 7


class _PairSumAddFn(torch.autograd.Function):
    """residual += pair sums of the gathered rows (in place); backward: the
    residual's gradient passes through and the rows get the row gradients."""

    @staticmethod
    def forward(ctx, residual, rows_var, dtable: DeviceTable, omap: OverlayMap, tokens, seg_start, t0: int,
                n: int, hit_count):
        dev = dtable.device
        nh, hpn, dim = dtable.n_heads, dtable.heads_per_ngram, dtable.dim
        if residual.dtype != torch.bfloat16 or not residual.is_contiguous() or tuple(residual.shape) != (n, hpn * dim):
            raise ValueError(f"residual must be contiguous bf16 [{n}, {hpn * dim}]")
        rv = rows_var.detach().contiguous()
        need_grad = rows_var.requires_grad and omap.R > 0
        slots = torch.empty(n, nh, dtype=torch.int32, device=dev) if need_grad else None
        _emit(dtable, omap, rv, tokens, seg_start, t0, n, L.MODE_PAIRSUM_ADD_BF16, residual, slots, hit_count)
        ctx.mark_dirty(residual)
        ctx.meta = (nh, hpn, dim, omap.R, n)
        ctx.peer = _peer_of(omap, rows_var)
        ctx.save_for_backward(slots if slots is not None else torch.empty(0, dtype=torch.int32, device=dev))
        return residual

    @staticmethod
    def backward(ctx, grad_res):
        (slots,) = ctx.saved_tensors
        nh, hpn, dim, R, n = ctx.meta
        grad_rows = None
        if ctx.needs_input_grad[1] and R > 0 and slots.numel():
            g = grad_res.contiguous().to(torch.bfloat16)
            if ctx.peer is not None:  # row gradients stored into their owners' receive buffers; no .grad
                ctx.peer.backward(slots, g, nh, hpn, L.MODE_PAIRSUM_ADD_BF16)
            else:
                grad_rows = row_gradients(slots, g, nh, hpn, dim, R, L.MODE_PAIRSUM_ADD_BF16)
        return (grad_res, grad_rows) + (None,) * 7


def _peer_of(omap: OverlayMap, rows_var: torch.Tensor):
    """The PeerRows attached to this overlay map (PeerRows.attach) when rows_var
    is its rows_var: the backward then hands the row gradients to it."""
    peer = getattr(omap, "peer", None)
    if peer is None or rows_var.data_ptr() != peer.rows_var.data_ptr():
        return None
    return peer


def row_gradients(slots: torch.Tensor, grad: torch.Tensor, n_heads: int, hpn: int, dim: int, R: int,
                  mode: int) -> torch.Tensor:
    """grad_rows [R, dim] from the saved slots (engram_backward): duplicates
    summed from +0 in ascending (t, h) order, bit-identical to the reference's
    index_put_(accumulate=True)."""
    dev = slots.device
    n = slots.shape[0]
    lib = L.load()
    ws_bytes = int(lib.engram_backward_workspace_bytes(n, n_heads, R))
    L.check(min(ws_bytes, 0), "engram_backward_workspace_bytes")
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
    out = torch.empty(R, dim, dtype=torch.float32, device=dev)
    st = lib.engram_backward(slots.data_ptr(), n, n_heads, hpn, mode, grad.data_ptr(), dim, R, out.data_ptr(),
                             ws.data_ptr(), ws_bytes, L.stream_of(dev))
    L.check(st, "engram_backward")
    return out


def engram_embed(dtable: DeviceTable, tokens, rows_var: torch.Tensor, omap: OverlayMap, seg_start=None,
                 t0: int = 0, n: int | None = None, hit_count: torch.Tensor | None = None) -> torch.Tensor:
    """emb [n, n_heads*dim] (fp32) of positions t0..t0+n-1, overlay substituted."""
    dev = dtable.device
    _check_rows_var(rows_var, dtable.dim)
    tokens = _as_i32(tokens, dev)
    if n is None:
        n = tokens.numel() - t0
    ss = None if seg_start is None else _as_i32(seg_start, dev)
    return _ConcatFn.apply(rows_var, dtable, omap, tokens, ss, t0, n, hit_count)


class _ConcatAtFn(torch.autograd.Function):
    """CONCAT rows at an explicit position list (decode-style)."""

    @staticmethod
    def forward(ctx, rows_var, dtable: DeviceTable, omap: OverlayMap, tokens, seg_start, positions, hit_count):
        dev = dtable.device
        nh, dim = dtable.n_heads, dtable.dim
        n = positions.numel()
        rv = rows_var.detach().contiguous()
        out = torch.empty(n, nh * dim, dtype=torch.float32, device=dev)
        need_grad = rows_var.requires_grad and omap.R > 0
        slots = torch.empty(n, nh, dtype=torch.int32, device=dev) if need_grad else None
        ov = omap.descriptor(rv)
        st = L.load().engram_forward_at(C.byref(dtable.ctable), C.byref(ov), tokens.data_ptr(), tokens.numel(),
                                        L.ptr(seg_start), positions.data_ptr(), n, L.MODE_CONCAT_F32, out.data_ptr(),
                                        None, L.ptr(slots), L.ptr(hit_count), L.stream_of(dev))
        L.check(st, "engram_forward_at")
        ctx.meta = (nh, dtable.heads_per_ngram, dim, omap.R, n)
        ctx.save_for_backward(slots if slots is not None else torch.empty(0, dtype=torch.int32, device=dev))
        return out

    @staticmethod
    def backward(ctx, grad_out):
        (slots,) = ctx.saved_tensors
        nh, hpn, dim, R, n = ctx.meta
        if not ctx.needs_input_grad[0] or R == 0 or slots.numel() == 0:
            return (None,) * 7
        grad_rows = row_gradients(slots, grad_out.contiguous().to(torch.float32), nh, hpn, dim, R, L.MODE_CONCAT_F32)
        return (grad_rows,) + (None,) * 6


def engram_embed_at(dtable: DeviceTable, tokens, positions, rows_var: torch.Tensor, omap: OverlayMap,
                    seg_start=None, hit_count: torch.Tensor | None = None) -> torch.Tensor:
    """emb [len(positions), n_heads*dim] for an explicit position list: the
    decode-style lookup (one new token per sequence; the reference computes it
    position by position with Replica.ple_true_emb, engraft/replica/model.py:473-495)."""
    dev = dtable.device
    _check_rows_var(rows_var, dtable.dim)
    tokens = _as_i32(tokens, dev)
    pos = torch.as_tensor(positions, dtype=torch.int64)
    if pos.numel() and (int(pos.min()) < 0 or int(pos.max()) >= tokens.numel()):
        raise ValueError("positions must lie in [0, len(tokens))")
    pos = pos.to(dev, non_blocking=True).contiguous()
    ss = None if seg_start is None else _as_i32(seg_start, dev)
    return _ConcatAtFn.apply(rows_var, dtable, omap, tokens, ss, pos, hit_count)


def engram_residual_add(residual: torch.Tensor, dtable: DeviceTable, tokens, rows_var: torch.Tensor,
                        omap: OverlayMap, seg_start=None, t0: int = 0,
                        hit_count: torch.Tensor | None = None) -> torch.Tensor:
    """residual[t, g*dim:(g+1)*dim] += row(g) + row(hpn+g), in place (bf16)."""
    dev = dtable.device
    _check_rows_var(rows_var, dtable.dim)
    tokens = _as_i32(tokens, dev)
    ss = None if seg_start is None else _as_i32(seg_start, dev)
    return _PairSumAddFn.apply(residual, rows_var, dtable, omap, tokens, ss, t0, residual.shape[0], hit_count)


_MAP_CACHE: dict = {}


def _overlay_map_for(row_map, device) -> OverlayMap:
    """The device map of a reference row_map ({global_id: index}).

    The descent builds row_map once per run and passes the same dict to every
    step (engraft/descend_corpus.py:776), so one map is built per (dict,
    device) and found again by the dict's identity and size in O(1): no
    per-build pass over its R items.  A dict changed in place without a change
    of size is not detected; after such a change call forget_overlay_map(row_map)
    (or pass a new dict).  An OverlayMap passed as row_map is used as it is."""
    if isinstance(row_map, OverlayMap):
        return row_map
    key = (id(row_map), str(device))
    hit = _MAP_CACHE.get(key)
    if hit is not None and hit[0] is row_map and hit[1] == len(row_map):
        return hit[2]
    omap = OverlayMap.from_row_map(row_map, device)
    if len(_MAP_CACHE) > 16:
        _MAP_CACHE.pop(next(iter(_MAP_CACHE)))
    _MAP_CACHE[key] = (row_map, len(row_map), omap)  # holds the dict, so its id is not recycled
    return omap


def forget_overlay_map(row_map=None) -> None:
    """Drops the cached device map of row_map (all cached maps when None), so
    the next build rebuilds it: needed after a dict is changed in place."""
    if row_map is None:
        _MAP_CACHE.clear()
        return
    for key in [k for k, v in _MAP_CACHE.items() if v[0] is row_map]:
        del _MAP_CACHE[key]


@dataclasses.dataclass
class OverlayEmb:
    """Drop-in for engraft.replica.seq.OverlayEmb (engraft/replica/seq.py:237-444).

    Same fields and `build(n_positions, start=0)`; the result lives on
    rows_var's device with rows_var's dtype (float32), shape
    [n_positions-start, n_heads*dim], differentiable in rows_var.  `table` is
    the reference's table object (made resident once per device) or a
    DeviceTable.  `row_map` is the reference's dict (its device map is built
    once per dict; see forget_overlay_map) or an OverlayMap.  `overlay_cache` is accepted for signature compatibility: the
    fused gather needs no per-fragment cache.  `n_id_hits` / `n_key_hits`
    count the (position, head) pairs served by the overlay, as in the
    reference."""

    table: object
    tokens: list
    rows_var: torch.Tensor
    row_map: dict
    segment_ids: torch.Tensor | None = None
    overlay_cache: dict | None = None

    def __post_init__(self) -> None:
        self._seg_start = None
        if self.segment_ids is not None:
            self._seg_start = seg_starts_from_segment_ids(self.segment_ids)
        self._hits = None
        self.n_key_hits = 0

    @property
    def n_id_hits(self) -> int:
        return 0 if self._hits is None else int(self._hits.item())

    def build(self, n_positions: int, start: int = 0) -> torch.Tensor:
        dev = self.rows_var.device
        if dev.type != "cuda":
            raise RuntimeError("engraft_ngram_b200.OverlayEmb runs on CUDA only: move rows_var to a CUDA device")
        dtable = DeviceTable.of(self.table, dev)
        _check_rows_var(self.rows_var, dtable.dim)
        if not (0 <= start <= n_positions <= len(self.tokens)):
            raise ValueError(f"build: need 0 <= start <= n_positions <= len(tokens), got {start}, {n_positions}")
        omap = _overlay_map_for(self.row_map, dev)
        if omap.R != self.rows_var.shape[0]:
            raise ValueError(f"rows_var has {self.rows_var.shape[0]} rows, row_map {omap.R}")
        toks = self.tokens[:n_positions]
        if isinstance(toks, torch.Tensor):
            toks = toks.to(torch.int64)
        else:
            toks = torch.from_numpy(np.asarray(toks, dtype=np.int64))
        if toks.numel() and (int(toks.max()) > 2**31 - 1 or int(toks.min()) < -2**31):
            raise ValueError("token id does not fit int32")
        toks = toks.to(torch.int32)
        if toks.device.type == "cpu":
            toks = toks.pin_memory()
        toks = toks.to(dev, non_blocking=True)
        ss = None
        if self._seg_start is not None:
            if len(self._seg_start) < n_positions:
                raise ValueError("segment_ids shorter than n_positions")
            ss = torch.from_numpy(self._seg_start[:n_positions]).to(dev, non_blocking=True)
        self._hits = torch.zeros(1, dtype=torch.int64, device=dev)
        return engram_embed(dtable, toks, self.rows_var, omap, ss, start, n_positions - start, self._hits)
