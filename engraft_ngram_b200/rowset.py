"""Row sets and overlay-file operations on the device.

Drop-ins for the set algebra around the descent, with the reference's arguments
and results:
- build_all_read_row_set (engraft/descend_corpus.py:1409-1430): the union of the
  rows every prefix position of every training fragment reads;
- build_rows_var (engraft/replica/distill.py:401-457): the sorted variable row
  set of a locality policy, minus the rows read at excluded positions, with
  its true rows;
- sum_overlays (engraft/replica/overlay_sum.py:36-112): the sum of the deltas
  of several .pleo files over the union of their rows, with its manifest;
- write_merged_pleo (engraft/descend_corpus.py:627-647): variable rows plus the
  frozen all-read rows at their true values.

A row set is a bitmap over the table's global rows (engram_rowset_*): hashing
the positions, the unions and differences and the sorted list all run on the
GPU; the true rows come from the resident table (engram_gather_rows).
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _lib as L
from .pleo import read_pleo, write_pleo
from .table import DeviceTable, _as_i32

OP_UNION, OP_DIFFERENCE, OP_INTERSECTION = 0, 1, 2
QUANT_FLOOR = 0.055  # recorded in the sum_overlays manifest, as the reference does
_POLICIES = ("all-read", "private", "entity", "t8-answer")


class DeviceRowSet:
    """A set of global rows of a table with n_rows rows, as a device bitmap."""

    def __init__(self, n_rows: int, device):
        lib = L.load()
        self.n_rows = int(n_rows)
        self.device = torch.device(device)
        self.words = int(lib.engram_rowset_words(self.n_rows))
        L.check(min(self.words, 0), "engram_rowset_words")
        self.bits = torch.zeros(max(self.words, 1), dtype=torch.int32, device=self.device)
        self._ws = None

    @classmethod
    def of_ids(cls, ids, n_rows: int, device) -> "DeviceRowSet":
        s = cls(n_rows, device)
        s.add_ids(ids)
        return s

    def add_ids(self, ids) -> "DeviceRowSet":
        ids = torch.as_tensor(np.asarray(ids, dtype=np.int64) if not torch.is_tensor(ids) else ids)
        if ids.numel() and (int(ids.min()) < 0 or int(ids.max()) >= self.n_rows):
            raise ValueError(f"row ids must lie in [0, {self.n_rows})")
        ids = ids.to(device=self.device, dtype=torch.int32).contiguous()
        st = L.load().engram_rowset_mark_ids(ids.data_ptr(), ids.numel(), self.n_rows, self.bits.data_ptr(),
                                             L.stream_of(self.device))
        L.check(st, "engram_rowset_mark_ids")
        self._ws = None
        return self

    def add_positions(self, table: DeviceTable, tokens, seg_start=None, positions=None) -> "DeviceRowSet":
        """Adds the rows of all heads at `positions` of `tokens` (all positions
        when None), each hashed with its context (RowSet.from_position,
        engraft/lens.py:127-136); seg_start[t] = first index of t's fragment."""
        tokens = _as_i32(tokens, self.device)
        ss = None if seg_start is None else _as_i32(seg_start, self.device)
        if positions is None:
            pos, n = None, tokens.numel()
        else:
            pos = torch.as_tensor(np.asarray(positions, dtype=np.int64) if not torch.is_tensor(positions)
                                  else positions).to(device=self.device, dtype=torch.int64).contiguous()
            n = pos.numel()
            if n and (int(pos.min()) < 0 or int(pos.max()) >= tokens.numel()):
                raise ValueError("positions must lie in [0, len(tokens))")
        if n == 0:
            return self
        st = L.load().engram_rowset_mark(C.byref(table.ctable), tokens.data_ptr(), tokens.numel(), L.ptr(ss),
                                         None if pos is None else pos.data_ptr(), n, self.bits.data_ptr(),
                                         L.stream_of(self.device))
        L.check(st, "engram_rowset_mark")
        self._ws = None
        return self

    def _combine(self, other: "DeviceRowSet", op: int) -> "DeviceRowSet":
        if other.n_rows != self.n_rows:
            raise ValueError("row sets over different tables")
        out = DeviceRowSet(self.n_rows, self.device)
        st = L.load().engram_rowset_combine(self.bits.data_ptr(), other.bits.data_ptr(), self.words, op,
                                            out.bits.data_ptr(), L.stream_of(self.device))
        L.check(st, "engram_rowset_combine")
        return out

    def __or__(self, other):
        return self._combine(other, OP_UNION)

    def __sub__(self, other):
        return self._combine(other, OP_DIFFERENCE)

    def __and__(self, other):
        return self._combine(other, OP_INTERSECTION)

    def _extract(self, capacity: int, out):
        lib = L.load()
        ws_bytes = int(lib.engram_rowset_workspace_bytes(self.words))
        L.check(min(ws_bytes, 0), "engram_rowset_workspace_bytes")
        if self._ws is None or self._ws.numel() < ws_bytes:
            self._ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=self.device)
        count = torch.zeros(1, dtype=torch.int64, device=self.device)
        st = lib.engram_rowset_extract(self.bits.data_ptr(), self.words, None if out is None else out.data_ptr(),
                                       capacity, count.data_ptr(), self._ws.data_ptr(), ws_bytes,
                                       L.stream_of(self.device))
        L.check(st, "engram_rowset_extract")
        return int(count.item())

    def __len__(self) -> int:
        return self._extract(0, None)

    def ids(self) -> torch.Tensor:
        """The members, ascending (int32 on the device)."""
        n = self._extract(0, None)
        out = torch.empty(max(n, 1), dtype=torch.int32, device=self.device)
        self._extract(n, out)
        return out[:n]

    def index(self, ids) -> torch.Tensor:
        """Position of each id in ids() (-1 for non-members), int32 on the device."""
        if self._ws is None:
            self._extract(0, None)
        ids = torch.as_tensor(ids).to(device=self.device, dtype=torch.int32).contiguous()
        out = torch.empty(max(ids.numel(), 1), dtype=torch.int32, device=self.device)
        st = L.load().engram_rowset_index(self.bits.data_ptr(), self.words, self._ws.data_ptr(), self._ws.numel(),
                                          ids.data_ptr(), ids.numel(), out.data_ptr(), L.stream_of(self.device))
        L.check(st, "engram_rowset_index")
        return out[: ids.numel()]


def _device(device):
    device = torch.device(device if device is not None else "cuda")
    if device.index is None:
        device = torch.device("cuda", torch.cuda.current_device())
    return device


def _fragments(frags) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Concatenated tokens, seg_start and the prefix positions (0..len-2 of
    each fragment) of a list of token lists."""
    lens = [len(f) for f in frags]
    total = sum(lens)
    tokens = np.zeros(total, dtype=np.int32)
    seg = np.zeros(total, dtype=np.int32)
    pos = []
    off = 0
    for f, n in zip(frags, lens):
        tokens[off:off + n] = np.asarray(f, dtype=np.int64).astype(np.int32)
        seg[off:off + n] = off
        if n > 1:
            pos.append(np.arange(off, off + n - 1, dtype=np.int64))
        off += n
    positions = np.concatenate(pos) if pos else np.zeros(0, dtype=np.int64)
    return tokens, seg, positions


def rows_read_by_prefixes(table, frags, device=None) -> DeviceRowSet:
    """The rows read by positions 0..len-2 of each token list in `frags`
    (_rows_read_by_prefix, engraft/descend_corpus.py:1409-1418, for all of them)."""
    dev = _device(device)
    t = DeviceTable.addressing_of(table, dev)
    s = DeviceRowSet(t.n_rows, dev)
    tokens, seg, positions = _fragments(frags)
    if positions.size:
        s.add_positions(t, tokens, seg, positions)
    return s


def build_all_read_row_set(table, train_frags_tokens, device=None) -> dict:
    """`{"all_read": [...]}` (ascending global rows), as the reference."""
    ids = rows_read_by_prefixes(table, train_frags_tokens, device).ids()
    return {"all_read": [int(g) for g in ids.cpu().numpy().tolist()]}


def _true_rows(table, ids: torch.Tensor, device) -> torch.Tensor:
    """Dequantised true rows of global ids (distill._read_true_rows,
    engraft/replica/distill.py:378-396), float32 [n, dim] on the device."""
    return DeviceTable.of(table, device).gather_rows(ids)


def build_rows_var(table, sequences, policy: str, row_sets: dict, exclude_positions: dict | None = None,
                   device=None, rows_on_device: bool = False):
    """`(row_map, rows_var)` as the reference: row_map {global row: index}
    in ascending global order, rows_var float32 [R, dim] of true rows (on the
    CPU like the reference, or on the device with rows_on_device=True)."""
    if policy not in _POLICIES:
        raise ValueError(f"build_rows_var: unknown policy {policy!r} (expected: {_POLICIES})")
    dev = _device(device)
    t = DeviceTable.addressing_of(table, dev)

    def rows_of(key: str) -> DeviceRowSet:
        return DeviceRowSet.of_ids(row_sets[key], t.n_rows, dev)

    if policy == "all-read":
        candidate = rows_of("all_read")
    elif policy == "private":
        candidate = rows_of("all_read") - rows_of("neutral_read")
    elif policy == "entity":
        candidate = rows_of("entity") | rows_of("terme")
    else:
        candidate = rows_of("t8_answer")
    excluded = DeviceRowSet(t.n_rows, dev)
    for seq_idx, positions in (exclude_positions or {}).items():
        if len(positions):
            excluded.add_positions(t, sequences[seq_idx], None, list(positions))
    selected = (candidate - excluded).ids()
    ids = selected.cpu().numpy()
    row_map = {int(g): i for i, g in enumerate(ids.tolist())}
    if ids.size == 0:
        dim = getattr(table, "dim", 160)
        return row_map, torch.zeros(0, dim, dtype=torch.float32, device=dev if rows_on_device else "cpu")
    rows = _true_rows(table, selected, dev)
    return row_map, (rows if rows_on_device else rows.cpu())


def _accumulate(acc: torch.Tensor, index: torch.Tensor, data: torch.Tensor, base: torch.Tensor) -> None:
    """acc[index[k]] += data[k] - base[k], repeated indices in file order: a
    stable device sort of the targets, then one launch that adds each run of
    equal targets in order (engram_overlay_accumulate with `order`)."""
    n = index.numel()
    if n == 0:
        return
    ix = index.contiguous()
    order = torch.sort(ix.long(), stable=True).indices.contiguous()
    d, b = data.contiguous(), base.contiguous()
    st = L.load().engram_overlay_accumulate(acc.data_ptr(), ix.data_ptr(), order.data_ptr(), d.data_ptr(),
                                            b.data_ptr(), n, acc.shape[1], L.stream_of(acc.device))
    L.check(st, "engram_overlay_accumulate")


def sum_overlays(table, pleo_paths: list, device=None):
    """`(rows_union, data_merged, manifest)` as the reference: the union of the
    files' rows (ascending int32), true rows + the float32 sum of each file's
    delta (rows - true rows), and the manifest of moved / shared rows."""
    if not pleo_paths:
        raise ValueError("sum_overlays: no .pleo files provided")
    dev = _device(device)
    t = DeviceTable.addressing_of(table, dev)
    files = [read_pleo(p) for p in pleo_paths]
    row_len = files[0][1].shape[1]
    union = DeviceRowSet(t.n_rows, dev)
    for rows, _ in files:
        union.add_ids(rows)
    rows_union = union.ids()
    n = rows_union.numel()
    delta_sum = torch.zeros(n, row_len, dtype=torch.float32, device=dev)
    moved_count = torch.zeros(n, dtype=torch.int64, device=dev)
    abs_sum = torch.zeros(n, dtype=torch.float64, device=dev)
    for rows, data in files:
        rows_d = torch.from_numpy(rows).to(dev)
        data_d = torch.from_numpy(data).to(dev)
        true_d = _true_rows(table, rows_d, dev)
        idx = union.index(rows_d)
        _accumulate(delta_sum, idx, data_d, true_d)
        norms = torch.linalg.vector_norm((data_d - true_d).to(torch.float64), dim=1)
        moved = norms > 0.0
        moved_count.index_add_(0, idx[moved].long(), torch.ones_like(idx[moved], dtype=torch.int64))
        abs_sum.index_add_(0, idx[moved].long(), norms[moved])
    true_union = _true_rows(table, rows_union, dev)
    data_merged = (true_union + delta_sum).cpu().numpy().astype(np.float32)
    sum_abs_norm = torch.linalg.vector_norm(delta_sum.to(torch.float64), dim=1).cpu().numpy()
    moved_count = moved_count.cpu().numpy()
    abs_sum = abs_sum.cpu().numpy()
    moved_any = moved_count >= 1
    shared = moved_count >= 2
    hist: dict[str, int] = {}
    for c in moved_count[moved_any].tolist():
        hist[str(int(c))] = hist.get(str(int(c)), 0) + 1
    ssa, sas = sum_abs_norm[shared], abs_sum[shared]
    max_norm = float(sum_abs_norm.max()) if n else 0.0
    manifest = {
        "n_files": len(pleo_paths),
        "n_rows_union": int(n),
        "n_rows_moved_any": int(moved_any.sum()),
        "n_rows_shared": int(shared.sum()),
        "facts_per_row_histogram": hist,
        "shared_rows_sum_abs_norm_mean": float(ssa.mean()) if ssa.size else None,
        "shared_rows_sum_abs_norm_max": float(ssa.max()) if ssa.size else None,
        "shared_rows_abs_sum_norm_mean": float(sas.mean()) if sas.size else None,
        "shared_rows_abs_sum_norm_max": float(sas.max()) if sas.size else None,
        "max_row_delta_norm": max_norm,
        "quant_floor": QUANT_FLOOR,
        "max_row_delta_norm_over_quant_floor": max_norm > QUANT_FLOOR,
    }
    return rows_union.cpu().numpy().astype(np.int32), data_merged, manifest


def write_merged_pleo(table, row_map: dict, rows_var: torch.Tensor, all_read_rows, out_path, device=None) -> dict:
    """Writes the variable rows (row_map order, current values) then the
    all-read rows that are not variable (ascending, true values), as the
    reference; returns {"n_rows_variable", "n_rows_frozen", "frozen_rows"}."""
    dev = _device(device)
    t = DeviceTable.addressing_of(table, dev)
    variable = DeviceRowSet.of_ids(list(row_map.keys()), t.n_rows, dev)
    frozen = (DeviceRowSet.of_ids(list(all_read_rows), t.n_rows, dev) - variable).ids()
    frozen_list = [int(g) for g in frozen.cpu().numpy().tolist()]
    rows_all = np.array(list(row_map.keys()) + frozen_list, dtype=np.int32)
    data_var = rows_var.detach().to("cpu", torch.float32).numpy()
    if frozen_list:
        data_frozen = _true_rows(table, frozen, dev).cpu().numpy()
        data_all = np.concatenate([data_var, data_frozen], axis=0) if data_var.shape[0] else data_frozen
    else:
        data_all = data_var
    write_pleo(out_path, rows_all, data_all)
    return {"n_rows_variable": len(row_map), "n_rows_frozen": len(frozen_list), "frozen_rows": frozen_list}
