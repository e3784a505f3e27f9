"""The Engram/PLE table resident in HBM.

`DeviceTable` keeps every row of the table on one GPU in the packed layout the
kernels read (see engram_table_pack in include/engram_b200.h) together with the
addressing constants of the reference's `PleTable` (engraft/table.py:40-88).
It also exposes the `PleTable` duck type (n_heads, heads_per_ngram, ngram_size,
eos_token_id, head_offsets, head_vocab_sizes, layer_multipliers,
ngram_addresses, read_rows) so reference code that only reads those keeps
working when handed a DeviceTable.
"""
from __future__ import annotations

import ctypes as C
import weakref

import numpy as np
import torch

from . import _lib as L


class DeviceTable:
    def __init__(self, rows: torch.Tensor, fmt: int, dim: int, head_sizes, head_offsets, mult, eos_token_id: int,
                 ngram_size: int = 3, heads_per_ngram: int = 8, n_rows: int | None = None, source=None,
                 hash_only: bool = False):
        """rows: uint8 CUDA tensor holding n_rows resident rows (engram_row_stride bytes each).
        hash_only=True: the table's addressing constants only (for hashing and
        scans); rows may be any small CUDA buffer and must never be gathered."""
        if not rows.is_cuda:
            raise RuntimeError("DeviceTable rows must live on a CUDA device")
        lib = L.load()
        stride = int(lib.engram_row_stride(fmt, dim))
        if stride < 0:
            L.check(stride, "engram_row_stride")
        self.rows = rows
        self.fmt = int(fmt)
        self.dim = int(dim)
        self.row_stride = stride
        self.n_rows = int(n_rows if n_rows is not None else rows.numel() // stride)
        self.hash_only = bool(hash_only)
        if not hash_only and rows.numel() < self.n_rows * stride:
            raise ValueError(f"rows holds {rows.numel()} bytes, need {self.n_rows * stride}")
        self.ngram_size = int(ngram_size)
        self.heads_per_ngram = int(heads_per_ngram)
        self.n_heads = (self.ngram_size - 1) * self.heads_per_ngram
        self.head_vocab_sizes = [int(x) for x in head_sizes]
        self.head_offsets = [int(x) for x in head_offsets]
        self.layer_multipliers = [int(x) for x in mult]
        self.eos_token_id = int(eos_token_id)
        self.source = source
        if len(self.head_vocab_sizes) != self.n_heads or len(self.head_offsets) != self.n_heads:
            raise ValueError(f"expected {self.n_heads} head sizes/offsets")
        sizes = np.asarray(self.head_vocab_sizes, dtype=np.int64)
        offs = np.asarray(self.head_offsets, dtype=np.int64)
        mu = np.asarray([m & 0xFFFFFFFFFFFFFFFF for m in self.layer_multipliers], dtype=np.uint64)
        self._ct = L.EngramTable()
        st = lib.engram_table_init(C.byref(self._ct), rows.data_ptr(), self.n_rows, self.fmt, self.dim,
                                   self.ngram_size, self.heads_per_ngram, sizes.ctypes.data, offs.ctypes.data,
                                   mu.ctypes.data, len(mu), self.eos_token_id)
        L.check(st, "engram_table_init")

    # ------------------------------------------------------------------ builders
    @property
    def device(self) -> torch.device:
        return self.rows.device

    @property
    def ctable(self) -> L.EngramTable:
        return self._ct

    @classmethod
    def from_raw(cls, raw, fmt: int, dim: int, head_sizes, head_offsets, mult, eos_token_id: int,
                 ngram_size: int = 3, heads_per_ngram: int = 8, device="cuda", source=None) -> "DeviceTable":
        """raw: the reference's row bytes (uint8 [n_rows, raw_row_bytes], numpy or
        torch; F32 tables may pass float32 [n_rows, dim]).  Uploaded and packed on
        the device by engram_table_pack."""
        lib = L.load()
        device = torch.device(device)
        if isinstance(raw, np.ndarray):
            raw = torch.from_numpy(np.ascontiguousarray(raw))
        n_rows = raw.shape[0]
        raw_u8 = raw.contiguous().view(torch.uint8).reshape(n_rows, -1)
        rb = int(lib.engram_raw_row_bytes(fmt, dim))
        L.check(min(rb, 0), "engram_raw_row_bytes")
        if raw_u8.shape[1] != rb:
            raise ValueError(f"raw rows have {raw_u8.shape[1]} bytes, format needs {rb}")
        stride = int(lib.engram_row_stride(fmt, dim))
        src = raw_u8.to(device, non_blocking=False)
        dst = torch.empty(n_rows * stride, dtype=torch.uint8, device=device)
        st = lib.engram_table_pack(fmt, dim, src.data_ptr(), n_rows, dst.data_ptr(), L.stream_of(device))
        L.check(st, "engram_table_pack")
        torch.cuda.current_stream(device).synchronize()
        del src
        return cls(dst, fmt, dim, head_sizes, head_offsets, mult, eos_token_id, ngram_size, heads_per_ngram,
                   n_rows=n_rows, source=source)

    @classmethod
    def from_reference(cls, table, device="cuda") -> "DeviceTable":
        """Makes a reference table object resident: a PleTable (per-head IQ4_NL
        GGUF; rows read once, head by head, with its own stripe reader
        engraft/table.py:90-104) or any object with read_rows (FakeTable,
        engraft/testing/fake_table.py:70-76; fp32 rows)."""
        if isinstance(table, DeviceTable):
            return table
        sizes = [int(x) for x in table.head_vocab_sizes]
        offs = [int(x) for x in table.head_offsets]
        n_rows = max(o + s for o, s in zip(offs, sizes))
        common = dict(head_sizes=sizes, head_offsets=offs, mult=list(table.layer_multipliers),
                      eos_token_id=int(table.eos_token_id), ngram_size=int(table.ngram_size),
                      heads_per_ngram=int(table.heads_per_ngram), device=device, source=table)
        if hasattr(table, "read_rows_raw"):
            raw = np.zeros((n_rows, 90), dtype=np.uint8)
            for h, (o, s) in enumerate(zip(offs, sizes)):
                raw[o:o + s] = table.read_rows_raw(h, 0, s)
            return cls.from_raw(raw, L.FMT_IQ4_NL, 160, **common)
        first = np.asarray(table.read_rows(0, 0, 1), dtype=np.float32)
        dim = first.shape[1]
        rows = np.zeros((n_rows, dim), dtype=np.float32)
        for h, (o, s) in enumerate(zip(offs, sizes)):
            rows[o:o + s] = table.read_rows(h, 0, s)
        return cls.from_raw(rows, L.FMT_F32, dim, **common)

    _registry: "weakref.WeakKeyDictionary" = weakref.WeakKeyDictionary()
    _addressing: "weakref.WeakKeyDictionary" = weakref.WeakKeyDictionary()

    @classmethod
    def addressing_of(cls, table, device) -> "DeviceTable":
        """A hash-only DeviceTable with a reference table's addressing constants
        (head sizes and offsets, multipliers, EOS, n-gram geometry), for hashing
        and corpus scans: no rows are read or uploaded.  Cached per (table
        object, device); a DeviceTable is returned as it is."""
        if isinstance(table, DeviceTable):
            return table
        device = torch.device(device)
        if device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        per = cls._addressing.setdefault(table, {})
        if device not in per:
            sizes = [int(x) for x in table.head_vocab_sizes]
            offs = [int(x) for x in table.head_offsets]
            per[device] = cls(torch.zeros(64, dtype=torch.uint8, device=device), L.FMT_F32, 4, sizes, offs,
                              list(table.layer_multipliers), int(table.eos_token_id),
                              ngram_size=int(table.ngram_size), heads_per_ngram=int(table.heads_per_ngram),
                              n_rows=max(o + s for o, s in zip(offs, sizes)), source=table, hash_only=True)
        return per[device]

    @classmethod
    def of(cls, table, device) -> "DeviceTable":
        """The resident copy of a reference table on `device`, built once per
        (table object, device) and cached for the object's lifetime."""
        if isinstance(table, DeviceTable):
            if table.device != torch.device(device):
                raise ValueError(f"DeviceTable lives on {table.device}, requested {device}")
            return table
        device = torch.device(device)
        if device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        per = cls._registry.setdefault(table, {})
        if device not in per:
            per[device] = cls.from_reference(table, device)
        return per[device]

    # -------------------------------------------------------------- operations
    def global_ids(self, tokens: torch.Tensor, seg_start: torch.Tensor | None = None, t0: int = 0,
                   n: int | None = None) -> torch.Tensor:
        """int32 [n, n_heads] global row ids (engram_hash)."""
        tokens = _as_i32(tokens, self.device)
        if n is None:
            n = tokens.numel() - t0
        ss = None if seg_start is None else _as_i32(seg_start, self.device)
        out = torch.empty(n, self.n_heads, dtype=torch.int32, device=self.device)
        st = L.load().engram_hash(C.byref(self._ct), tokens.data_ptr(), L.ptr(ss), t0, n, out.data_ptr(),
                                  L.stream_of(self.device))
        L.check(st, "engram_hash")
        return out

    def ngram_addresses(self, tokens: list[int]) -> list[list[int]]:
        """Same contract as PleTable.ngram_addresses (engraft/table.py:111-144):
        local indices per position, computed on the GPU."""
        if len(tokens) == 0:
            return []
        ids = self.global_ids(torch.tensor(tokens, dtype=torch.int32)).to(torch.int64).cpu()
        ids -= torch.tensor(self.head_offsets, dtype=torch.int64)
        return ids.tolist()

    def gather_rows(self, ids) -> torch.Tensor:
        """float32 [n, dim] dequantised rows by global id (engram_gather_rows)."""
        if self.hash_only:
            raise RuntimeError("this DeviceTable holds addressing constants only (hash_only=True)")
        ids = _as_i32(ids, self.device).reshape(-1)
        if ids.numel():
            lo, hi = int(ids.min()), int(ids.max())
            if lo < 0 or hi >= self.n_rows:
                raise ValueError(f"row id outside [0, {self.n_rows})")
        out = torch.empty(ids.numel(), self.dim, dtype=torch.float32, device=self.device)
        st = L.load().engram_gather_rows(C.byref(self._ct), ids.data_ptr(), ids.numel(), out.data_ptr(),
                                         L.stream_of(self.device))
        L.check(st, "engram_gather_rows")
        return out

    def read_rows(self, h: int, start: int, n: int) -> np.ndarray:
        """PleTable.read_rows duck type (engraft/table.py:106-109): float32 [n, dim]."""
        if not (0 <= start and start + n <= self.head_vocab_sizes[h]):
            raise AssertionError(f"head {h}: requested rows [{start},{start + n}) outside [0,{self.head_vocab_sizes[h]})")
        ids = torch.arange(start, start + n, dtype=torch.int32) + self.head_offsets[h]
        return self.gather_rows(ids).cpu().numpy()


def _as_i32(x, device) -> torch.Tensor:
    if isinstance(x, torch.Tensor):
        t = x
    else:
        t = torch.as_tensor(np.asarray(x), dtype=torch.int32)
    if t.dtype != torch.int32:
        if t.numel() and (int(t.max()) > 2**31 - 1 or int(t.min()) < -2**31):
            raise ValueError("token/row id does not fit int32")
        t = t.to(torch.int32)
    return t.to(device, non_blocking=True).contiguous()


def synthetic_resident(n_rows: int, fmt: int, dim: int, seed: int, device, sigma: float = 1e-3,
                       f32_sigma: float = 0.0085, out: torch.Tensor | None = None) -> torch.Tensor:
    """Seeded synthetic table generated directly in the resident layout on the
    device (the full-size tables do not pass through host memory).  IQ4 rows:
    uniform random nibbles and sub-scales, fp16 block scales |N(0, sigma)|;
    F32 rows ~N(0, f32_sigma^2).  out: a uint8 buffer of at least
    n_rows * stride bytes to fill (e.g. a shard in symmetric memory)."""
    lib = L.load()
    stride = int(lib.engram_row_stride(fmt, dim))
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    if out is not None:
        if out.numel() < n_rows * stride:
            raise ValueError("synthetic_resident: out is too small")
        out = out.reshape(-1)[: n_rows * stride].view(n_rows, stride)
    if fmt == L.FMT_F32:
        t = torch.randn(n_rows, dim, generator=g, device=device, dtype=torch.float32) * f32_sigma
        if out is not None:
            out.copy_(t.view(torch.uint8).reshape(n_rows, stride))
            return out.reshape(-1)
        return t.view(torch.uint8).reshape(-1)
    if out is None:
        out = torch.empty(n_rows, stride, dtype=torch.uint8, device=device)
    chunk = 1 << 24
    for lo in range(0, n_rows, chunk):
        hi = min(n_rows, lo + chunk)
        blk = out[lo:hi]
        blk.random_(0, 256, generator=g)
        if fmt == L.FMT_IQ4_NL:
            nb = dim // 32
            d = (torch.randn(hi - lo, nb, generator=g, device=device) * sigma).abs().to(torch.float16)
            blk[:, 16 * nb:18 * nb] = d.view(torch.uint8).reshape(hi - lo, 2 * nb)
            blk[:, 18 * nb:] = 0
        else:
            ns = dim // 256
            v = blk.view(hi - lo, ns, 144)
            d = (torch.randn(hi - lo, ns, generator=g, device=device) * sigma).abs().to(torch.float16)
            v[:, :, 128:130] = d.view(torch.uint8).reshape(hi - lo, ns, 2)
            v[:, :, 136:] = 0
    return out.reshape(-1)


def synthetic_head_sizes(total_rows: int, n_heads: int = 16) -> list[int]:
    """Near-equal head sizes summing to total_rows; none a power of two."""
    base = total_rows // n_heads
    sizes = [base - (7 * (n_heads - 1 - h)) for h in range(n_heads)]
    sizes[-1] += total_rows - sum(sizes)
    for s in sizes:
        assert s > 0 and (s & (s - 1)) != 0
    return sizes


def synthetic_multipliers(seed: int, ngram_size: int = 3) -> list[int]:
    rng = np.random.default_rng(seed)
    return [int(x) | 1 for x in rng.integers(1, 2**63, size=ngram_size + 1, dtype=np.uint64)]
