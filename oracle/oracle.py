"""ctypes wrapper of the CPU oracle (engram_oracle.c).

TEST INFRASTRUCTURE ONLY: the checker for the CUDA path.  Imported by tests/,
__graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference leg;
never by the product package.  Each function names the reference code that the
C restatement follows (paths inside the fulvian/engraft-ngram project).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"

FMT_F32, FMT_IQ4_NL, FMT_IQ4_XS = 0, 1, 2
MODE_CONCAT_F32, MODE_PAIRSUM_ADD_BF16 = 0, 1

_lib = None


def build() -> Path:
    """Compile liboracle.so with the committed Makefile (gcc)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        src = HERE / "engram_oracle.c"
        if not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < src.stat().st_mtime:
            build()
        L = C.CDLL(str(LIB_PATH))
        p, i32, i64, u64p = C.c_void_p, C.c_int32, C.c_int64, C.c_void_p
        L.orc_hash.argtypes = [p, p, i64, i64, i32, i32, u64p, p, p, i64, p]
        L.orc_hash.restype = None
        L.orc_raw_row_bytes.argtypes = [i32, i32]
        L.orc_raw_row_bytes.restype = i64
        L.orc_dequant.argtypes = [i32, i32, p, i64, p]
        L.orc_dequant.restype = None
        L.orc_forward.argtypes = [i32, i32, p, i64, p, i64, i32, i32, p, p, p, i64, i32, p, p]
        L.orc_forward.restype = None
        L.orc_backward.argtypes = [p, i64, i32, i32, i32, p, i32, i64, p]
        L.orc_backward.restype = None
        L.orc_adam.argtypes = [p, p, p, p, p, i64, i64, C.c_double, C.c_double, C.c_double, C.c_double, C.c_float]
        L.orc_adam.restype = None
        L.orc_pack.argtypes = [i32, i32, p, i64, p, i64]
        L.orc_pack.restype = None
        L.orc_num_threads.restype = C.c_int
        L.orc_set_num_threads.argtypes = [C.c_int]
        _lib = L
    return _lib


def _ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def set_num_threads(n: int) -> None:
    lib().orc_set_num_threads(int(n))


def num_threads() -> int:
    return int(lib().orc_num_threads())


def raw_row_bytes(fmt: int, dim: int) -> int:
    return int(lib().orc_raw_row_bytes(fmt, dim))


def resident_row_bytes(fmt: int, dim: int) -> int:
    """Bytes per row of the device-resident layout (the C ABI's engram_row_stride)."""
    if fmt == FMT_F32:
        return dim * 4
    if fmt == FMT_IQ4_NL:
        return ((dim // 32) * 18 + 15) // 16 * 16
    return (dim // 256) * 144


def hash_ids(tokens, ngram_size, hpn, mult, head_sizes, head_offsets, eos, seg_start=None, t0=0, n=None):
    """Global row ids [n, n_heads] of positions t0..t0+n-1 (engraft/table.py:111-144,
    global ids per engraft/lens.py:108-110; segments per engraft/replica/seq.py:393-399)."""
    tokens = np.ascontiguousarray(tokens, dtype=np.int32)
    if n is None:
        n = tokens.shape[0] - t0
    n_heads = (ngram_size - 1) * hpn
    out = np.empty((n, n_heads), dtype=np.int32)
    if n == 0:
        return out
    m = np.zeros(8, dtype=np.uint64)
    m[:len(mult)] = np.asarray([int(x) for x in mult], dtype=np.uint64)
    sizes = np.ascontiguousarray(head_sizes, dtype=np.int64)
    offs = np.ascontiguousarray(head_offsets, dtype=np.int64)
    ss = None if seg_start is None else np.ascontiguousarray(seg_start, dtype=np.int32)
    lib().orc_hash(_ptr(tokens), _ptr(ss), t0, n, ngram_size, hpn, _ptr(m), _ptr(sizes), _ptr(offs),
                   int(eos), _ptr(out))
    return out


def dequant(fmt: int, dim: int, raw) -> np.ndarray:
    """float32 [n, dim] from the reference's raw row bytes (engraft/table.py:147-169,
    engraft/replica/dequant.py:127-189)."""
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    n = raw.shape[0]
    out = np.empty((n, dim), dtype=np.float32)
    if n:
        lib().orc_dequant(fmt, dim, _ptr(raw), n, _ptr(out))
    return out


def forward(fmt, dim, table_raw, ids, hpn, ov_rows, ov_ids, mode=MODE_CONCAT_F32, residual=None):
    """OverlayEmb.build on rows (engraft/replica/seq.py:372-444).  Returns
    (out, slots): CONCAT -> float32 [n, n_heads, dim]; PAIRSUM_ADD_BF16 ->
    uint16 (bf16 bits) [n, hpn*dim] = residual + pair sums.  ov_ids[k] is the
    global id of overlay row k (row_map = {ov_ids[k]: k})."""
    table_raw = np.ascontiguousarray(table_raw, dtype=np.uint8)
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    n, n_heads = ids.shape
    ov_rows = np.ascontiguousarray(ov_rows, dtype=np.float32).reshape(-1, dim)
    ov_ids = np.asarray(ov_ids, dtype=np.int32)
    order = np.argsort(ov_ids, kind="stable")
    keys = np.ascontiguousarray(ov_ids[order])
    vals = np.ascontiguousarray(order.astype(np.int32))
    slots = np.empty((n, n_heads), dtype=np.int32)
    if mode == MODE_CONCAT_F32:
        out = np.empty((n, n_heads, dim), dtype=np.float32)
    else:
        out = np.array(residual, dtype=np.uint16, copy=True).reshape(n, hpn * dim)
    if n:
        lib().orc_forward(fmt, dim, _ptr(table_raw), table_raw.shape[0], _ptr(ids), n, n_heads, hpn,
                          _ptr(ov_rows), _ptr(keys), _ptr(vals), keys.shape[0], mode, _ptr(out), _ptr(slots))
    return out, slots


def backward(slots, hpn, grad, dim, R, mode=MODE_CONCAT_F32) -> np.ndarray:
    """Row gradients [R, dim], duplicates summed from +0 in ascending (t,h)
    order (autograd of engraft/replica/seq.py:433-441)."""
    slots = np.ascontiguousarray(slots, dtype=np.int32)
    n, n_heads = slots.shape
    if mode == MODE_CONCAT_F32:
        grad = np.ascontiguousarray(grad, dtype=np.float32)
    else:
        grad = np.ascontiguousarray(grad, dtype=np.uint16)
    out = np.empty((R, dim), dtype=np.float32)
    lib().orc_backward(_ptr(slots), n, n_heads, hpn, mode, _ptr(grad), dim, R, _ptr(out))
    return out


def adam_(p, g, m, v, step, lr, beta1=0.9, beta2=0.999, eps=1e-8, p0=None, reg_scale=0.0) -> None:
    """In-place Adam step with the descent's regulariser gradient
    (engraft/descend_corpus.py:921-947; torch.optim.Adam single-tensor rule)."""
    for a in (p, m, v):
        assert a.dtype == np.float32 and a.flags.c_contiguous
    g = np.ascontiguousarray(g, dtype=np.float32)
    p0c = None if p0 is None else np.ascontiguousarray(p0, dtype=np.float32)
    lib().orc_adam(_ptr(p), _ptr(g), _ptr(m), _ptr(v), _ptr(p0c), p.size, int(step), float(lr),
                   float(beta1), float(beta2), float(eps), float(np.float32(reg_scale)))


def reg_scale(mu: float, rows0) -> np.float32:
    """float(mu) / max(sum(p0^2), 1e-12) in fp32, the factor autograd applies to
    2*(p-p0) (engraft/descend_corpus.py:936).  The sum is taken in float64 then
    rounded; torch's own fp32 reduction order may differ in the last bit."""
    S = np.float32(max(float(np.square(np.asarray(rows0, dtype=np.float64)).sum()), 1e-12))
    return np.float32(np.float32(mu) / S)


def pack(fmt: int, dim: int, raw) -> np.ndarray:
    """Reference raw rows -> device-resident row layout (uint8 [n, stride])."""
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    n = raw.shape[0]
    stride = resident_row_bytes(fmt, dim)
    out = np.empty((n, stride), dtype=np.uint8)
    if n:
        lib().orc_pack(fmt, dim, _ptr(raw), n, _ptr(out), stride)
    return out


def bf16_bits(x) -> np.ndarray:
    """float32 -> bf16 bit patterns, round to nearest even (uint16)."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (b & 0x7FFFFFFF) > 0x7F800000
    r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((b[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_to_f32(bits) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def scan_hits(tokens, ngram_size, hpn, mult, head_sizes, head_offsets, eos, overlay_sorted, dnorm_sorted) -> dict:
    """engraft/damage.py:168-224 restated: hit positions of the overlay rows and
    per-row read counts (dict with the reference's keys)."""
    L = lib()
    if not hasattr(L, "_scan_typed"):
        p, i32, i64 = C.c_void_p, C.c_int32, C.c_int64
        L.orc_scan_hits.argtypes = [p, i64, i32, i32, p, p, p, i64, p, p, i64, p, p, p, p, p]
        L.orc_scan_hits.restype = i64
        L._scan_typed = True
    tokens = np.ascontiguousarray(tokens, dtype=np.int32)
    n = tokens.shape[0]
    ov = np.ascontiguousarray(overlay_sorted, dtype=np.int32)
    dn = np.ascontiguousarray(dnorm_sorted, dtype=np.float32)
    m = np.zeros(8, dtype=np.uint64)
    m[:len(mult)] = np.asarray([int(x) for x in mult], dtype=np.uint64)
    sizes = np.ascontiguousarray(head_sizes, dtype=np.int64)
    offs = np.ascontiguousarray(head_offsets, dtype=np.int64)
    pos = np.empty(max(n, 1), np.int64)
    nh = np.empty(max(n, 1), np.int32)
    dmax = np.empty(max(n, 1), np.float32)
    dsum = np.empty(max(n, 1), np.float32)
    rc = np.empty(max(len(ov), 1), np.int64)
    k = L.orc_scan_hits(_ptr(tokens), n, ngram_size, hpn, _ptr(m), _ptr(sizes), _ptr(offs), int(eos), _ptr(ov),
                        _ptr(dn), len(ov), _ptr(pos), _ptr(nh), _ptr(dmax), _ptr(dsum), _ptr(rc))
    return {"pos": pos[:k], "n_hit_rows": nh[:k], "dnorm_max": dmax[:k], "dnorm_sum": dsum[:k],
            "read_count": rc[:len(ov)], "n_tokens": n}


# ---------------------------------------------------------------- row sets
def rows_read_by_prefixes(frags, ngram_size, hpn, mult, head_sizes, head_offsets, eos) -> np.ndarray:
    """Ascending global rows read by positions 0..len-2 of each token list
    (engraft/descend_corpus.py:1409-1430: _rows_read_by_prefix for every
    fragment, then the sorted union)."""
    parts = []
    for f in frags:
        f = np.asarray(f, dtype=np.int64).astype(np.int32)
        if f.size > 1:
            parts.append(hash_ids(f, ngram_size, hpn, mult, head_sizes, head_offsets, eos)[: f.size - 1].ravel())
    return np.unique(np.concatenate(parts)) if parts else np.zeros(0, np.int32)


def rows_var_ids(policy, sets, sequences, exclude_positions, ngram_size, hpn, mult, head_sizes, head_offsets,
                 eos) -> np.ndarray:
    """The ascending variable rows of build_rows_var (engraft/replica/distill.py:401-457):
    the policy's set algebra over the census lists, minus every row read at an
    excluded position (all heads)."""
    a = lambda k: np.unique(np.asarray(sets[k], dtype=np.int64))  # noqa: E731
    if policy == "all-read":
        cand = a("all_read")
    elif policy == "private":
        cand = np.setdiff1d(a("all_read"), a("neutral_read"))
    elif policy == "entity":
        cand = np.union1d(a("entity"), a("terme"))
    elif policy == "t8-answer":
        cand = a("t8_answer")
    else:
        raise ValueError(policy)
    excl = []
    for s, positions in (exclude_positions or {}).items():
        toks = np.asarray(sequences[s], dtype=np.int64).astype(np.int32)
        ids = hash_ids(toks, ngram_size, hpn, mult, head_sizes, head_offsets, eos)
        excl.append(ids[np.asarray(positions, dtype=np.int64)].ravel())
    if excl:
        cand = np.setdiff1d(cand, np.concatenate(excl))
    return cand.astype(np.int32)


def sum_overlays(files, true_rows_of):
    """engraft/replica/overlay_sum.py:36-112 restated: files = [(rows, data)];
    true_rows_of(ids) -> float32 [n, dim].  Returns (rows_union, data_merged,
    counts) with counts = (moved_any, shared, histogram dict)."""
    union = np.unique(np.concatenate([np.asarray(r, dtype=np.int64) for r, _ in files])).astype(np.int32)
    n, dim = union.size, files[0][1].shape[1]
    delta_sum = np.zeros((n, dim), dtype=np.float32)
    moved = np.zeros(n, dtype=np.int64)
    for rows, data in files:
        delta = data.astype(np.float32) - true_rows_of(rows).astype(np.float32)
        idx = np.searchsorted(union, rows)
        np.add.at(delta_sum, idx, delta)
        np.add.at(moved, idx[np.any(delta != 0, axis=1)], 1)
    merged = (true_rows_of(union).astype(np.float32) + delta_sum).astype(np.float32)
    hist = {}
    for c in moved[moved >= 1].tolist():
        hist[str(c)] = hist.get(str(c), 0) + 1
    return union, merged, (int((moved >= 1).sum()), int((moved >= 2).sum()), hist)


def ple_forward(emb, hidden, w_key, w_value, norm_key, norm_query, norm_conv, conv1d, hist, hc, n_embd, eps,
                dilation):
    """The PLE block restated in float32 numpy (engraft/replica/layers.py:565-626,
    with rmsnorm layers.py:23-42 and causal_depthwise_conv layers.py:257-293):
    key/value projections, grouped RMS norms, the sign-sqrt sigmoid gate, the
    gated value's norm, the causal dilated depthwise conv over [history; T] and
    silu; returns (hidden + gated + conv, the last (K-1)*dilation rows of
    [history; normed])."""
    T = emb.shape[0]

    def rms(x, w):
        ms = (x * x).mean(axis=-1, keepdims=True, dtype=np.float32)
        return (x * (1.0 / np.sqrt(ms + np.float32(eps)))) * w.reshape(hc, n_embd)

    key = (emb @ w_key.T).reshape(T, hc, n_embd)
    s = (rms(key, norm_key) * rms(hidden, norm_query)).sum(axis=-1, dtype=np.float32) / np.float32(np.sqrt(n_embd))
    mag = np.sqrt(np.maximum(np.abs(s), np.float32(1e-6)))
    gate = (1.0 / (1.0 + np.exp(-(np.sign(s) * mag)))).astype(np.float32)
    value = emb @ w_value.T
    gated = value[:, None, :] * gate[:, :, None]
    normed = rms(gated, norm_conv)
    C = hc * n_embd
    full = np.concatenate([hist.reshape(-1, C), normed.reshape(T, C)]).astype(np.float32)
    H = hist.shape[0]
    K = conv1d.shape[1]
    acc = np.zeros((T, C), dtype=np.float32)
    for k in range(K):
        back = (K - 1 - k) * dilation
        for t in range(T):
            if H + t - back >= 0:
                acc[t] += full[H + t - back] * conv1d[:, k]
    conv = (acc / (1.0 + np.exp(-acc))).astype(np.float32).reshape(T, hc, n_embd)
    out = (hidden + gated + conv).astype(np.float32)
    hist_len = (K - 1) * dilation
    new_hist = np.concatenate([hist, normed])[-hist_len:] if hist_len > 0 else normed[:0]
    return out, new_hist.astype(np.float32)
