"""Bulk hash + overlay hit scan over a token corpus on the GPU: the drop-in for
engraft.damage.scan_hits (engraft/damage.py:168-224).

Same arguments and result: for every position of `tokens` whose 16 rows include
an overlay row (the corpus's last position excluded), its position, the number
of overlay rows it reads, and the max / float32 pairwise sum of their dnorm;
per overlay row, how many times it is read.  The corpus streams through the GPU
in blocks with 2 tokens of overlap (engraft/damage.py:107-121), so a corpus
larger than device memory scans in one pass.
"""
from __future__ import annotations

import ctypes as C
import time

import numpy as np
import torch

from . import _lib as L
from .overlay import OverlayMap
from .table import DeviceTable

BLOCK_TOKENS = 8_000_000


def scan_hits(tokens, table, overlay_sorted, dnorm_sorted, block: int = BLOCK_TOKENS, device=None) -> dict:
    """`table`: a DeviceTable, or the reference's table object (PleTable,
    FakeTable), of which only the addressing constants are used."""
    lib = L.load()
    if not isinstance(table, DeviceTable):
        table = DeviceTable.addressing_of(table, device if device is not None else "cuda")
    dev = table.device
    stream = L.stream_of(dev)
    tokens = np.asarray(tokens)
    n = int(tokens.shape[0])
    ov_sorted = np.asarray(overlay_sorted, dtype=np.int64)
    if ov_sorted.size and (np.any(np.diff(ov_sorted) <= 0) or ov_sorted.min() < 0 or ov_sorted.max() > 2**31 - 1):
        raise ValueError("overlay_sorted must be strictly increasing int32 row ids")
    R = int(ov_sorted.shape[0])
    omap = OverlayMap(torch.from_numpy(ov_sorted.astype(np.int32)), dev)
    ov = L.EngramOverlay(None, R, omap.keys.data_ptr() if R else None, omap.slots.data_ptr() if R else None,
                         omap.capacity)
    dnorm = torch.from_numpy(np.ascontiguousarray(dnorm_sorted, dtype=np.float32)).to(dev)
    read_count = torch.zeros(max(R, 1), dtype=torch.int64, device=dev)
    cap = min(n, block) + 2
    ws_bytes = int(lib.engram_scan_hits_workspace_bytes(cap))
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
    pos = torch.empty(max(cap, 1), dtype=torch.int64, device=dev)
    nhit = torch.empty(max(cap, 1), dtype=torch.int32, device=dev)
    dmax = torch.empty(max(cap, 1), dtype=torch.float32, device=dev)
    dsum = torch.empty(max(cap, 1), dtype=torch.float32, device=dev)
    n_hits = torch.zeros(1, dtype=torch.int64, device=dev)
    parts = {k: [] for k in ("pos", "n_hit_rows", "dnorm_max", "dnorm_sum")}
    torch.cuda.synchronize(dev)
    t_start = time.time()
    offset = 0
    while offset < n:
        this = min(block, n - offset)
        lo = offset if offset == 0 else offset - 2
        blk = torch.from_numpy(np.ascontiguousarray(tokens[lo:offset + this], dtype=np.int32)).to(dev)
        t0 = offset - lo
        last = offset + this >= n
        st = lib.engram_scan_hits(C.byref(table.ctable), blk.data_ptr(), t0, this, lo, 1 if last else 0, C.byref(ov),
                                  dnorm.data_ptr() if R else None, pos.data_ptr(), nhit.data_ptr(), dmax.data_ptr(),
                                  dsum.data_ptr(), n_hits.data_ptr(), read_count.data_ptr() if R else None,
                                  ws.data_ptr(), ws_bytes, stream)
        L.check(st, "engram_scan_hits")
        k = int(n_hits.item())
        parts["pos"].append(pos[:k].cpu().numpy())
        parts["n_hit_rows"].append(nhit[:k].cpu().numpy())
        parts["dnorm_max"].append(dmax[:k].cpu().numpy())
        parts["dnorm_sum"].append(dsum[:k].cpu().numpy())
        offset += this
    dt = time.time() - t_start

    def cat(key, dtype):
        return np.concatenate(parts[key]) if parts[key] else np.zeros(0, dtype=dtype)

    return {"pos": cat("pos", np.int64), "n_hit_rows": cat("n_hit_rows", np.int32),
            "dnorm_max": cat("dnorm_max", np.float32), "dnorm_sum": cat("dnorm_sum", np.float32),
            "read_count": read_count[:R].cpu().numpy(), "scan_time_s": dt, "n_tokens": n}
