""".pleo overlay files (engraft/lens.py:33-59): magic "PLEO", u32 n, u32 dim,
<i4 rows[n], <f4 data[n*dim], all little-endian.

The reference fixes dim = 160 (engraft/lens.py:38-39); these functions keep its
byte layout and accept any dim, with `strict_160=True` reproducing the
reference's check.  `read_pleo_device` loads an overlay straight into the
(row_map, rows_var) pair the CUDA path consumes.
"""
from __future__ import annotations

import struct
from pathlib import Path

import numpy as np

PLEO_MAGIC = b"PLEO"


def write_pleo(path, rows_global, data, strict_160: bool = False) -> None:
    rows = np.asarray(rows_global, dtype="<i4")
    values = np.asarray(data, dtype="<f4")
    if rows.ndim != 1:
        raise ValueError(f"rows_global must be 1-D, got ndim={rows.ndim}")
    n = rows.shape[0]
    if values.ndim != 2 or values.shape[0] != n or (strict_160 and values.shape[1] != 160):
        want = f"({n}, 160)" if strict_160 else f"({n}, dim)"
        raise ValueError(f"data.shape={values.shape}, expected {want}")
    with open(path, "wb") as f:
        f.write(PLEO_MAGIC)
        f.write(struct.pack("<II", n, values.shape[1]))
        f.write(rows.tobytes())
        f.write(values.tobytes())


def read_pleo(path) -> tuple[np.ndarray, np.ndarray]:
    with open(path, "rb") as f:
        magic = f.read(4)
        if magic != PLEO_MAGIC:
            raise ValueError(f"bad magic: {magic!r}, expected {PLEO_MAGIC!r}")
        n, dim = struct.unpack("<II", f.read(8))
        rows = np.frombuffer(f.read(n * 4), dtype="<i4").astype(np.int32).copy()
        data = np.frombuffer(f.read(n * dim * 4), dtype="<f4").astype(np.float32).copy()
    if rows.shape[0] != n or data.shape[0] != n * dim:
        raise ValueError(f"truncated .pleo file {path}")
    return rows, data.reshape(n, dim)


def read_pleo_device(path, device):
    """(row_map {global_id: index}, rows_var float32 [n, dim] on `device`), rows
    sorted ascending like build_rows_var (engraft/replica/distill.py:452-457)."""
    import torch
    rows, data = read_pleo(path)
    order = np.argsort(rows, kind="stable")
    rows, data = rows[order], data[order]
    row_map = {int(g): i for i, g in enumerate(rows.tolist())}
    return row_map, torch.from_numpy(data).to(device)
