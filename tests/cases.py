"""Rebuilds the inputs of each golden overlay case (tests/golden) so the oracle
and the CUDA path can be run on exactly the data the reference saw."""
from __future__ import annotations

import dataclasses
import hashlib

import numpy as np

import fixtures as FX
from oracle import oracle as O


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@dataclasses.dataclass
class TableSpec:
    fmt: int
    dim: int
    raw: np.ndarray          # reference raw row bytes [n_rows, raw_row_bytes]
    params: dict             # mult, head_sizes, head_offsets, eos, ngram_size, hpn

    @property
    def n_heads(self) -> int:
        return (self.params["ngram_size"] - 1) * self.params["hpn"]

    def ids(self, tokens, seg_start=None, t0=0, n=None):
        p = self.params
        return O.hash_ids(tokens, p["ngram_size"], p["hpn"], p["mult"], p["head_sizes"], p["head_offsets"],
                          p["eos"], seg_start=seg_start, t0=t0, n=n)

    def true_rows(self, ids) -> np.ndarray:
        return O.dequant(self.fmt, self.dim, self.raw[np.asarray(ids, dtype=np.int64)])


def syn_table() -> TableSpec:
    return TableSpec(O.FMT_IQ4_NL, 160, FX.syn_table_raw(), FX.syn_params())


def fake_table(rows_f32: np.ndarray, seed: int = 1) -> TableSpec:
    return TableSpec(O.FMT_F32, 160, rows_f32.view(np.uint8).reshape(rows_f32.shape[0], -1),
                     FX.fake_table_params(seed=seed))


@dataclasses.dataclass
class OverlayCase:
    table: TableSpec
    tokens: np.ndarray
    seg_start: np.ndarray | None
    t0: int
    n: int
    row_ids: np.ndarray
    rows_init: np.ndarray
    grad: np.ndarray
    golden: dict


def overlay_case(golden, prefix: str, table: TableSpec) -> OverlayCase:
    g = {k[len(prefix):]: golden[k] for k in golden.files if k.startswith(prefix)}
    tokens = g["tokens"]
    n_prefix = int(g["n_prefix"])
    start = int(g["start"])
    seg_start = FX.seg_starts(g["segment_ids"]) if int(g["use_segments"]) else None
    row_ids = g["row_ids"]
    rows_init = (table.true_rows(row_ids) + FX.overlay_noise(int(g["seed"]), (len(row_ids), table.dim))).astype(np.float32)
    assert sha(rows_init) == str(g["rows_init_sha"]), "fixture regeneration drifted from the reference's inputs"
    n = n_prefix - start
    grad = FX.overlay_grad(int(g["seed"]), (n, table.n_heads * table.dim))
    return OverlayCase(table, tokens, seg_start, start, n, row_ids, rows_init, grad, g)


def shard_plan_ref(ids, ov_ids, world: int, rank: int):
    """The contract of engram_shard_plan restated in numpy (a test reference):
    the pairs of `ids` (global row ids [n, n_heads]) whose owner id % world is
    another rank and which the overlay (ov_ids) does not serve are requested;
    send_ids holds each such id once, grouped by owner (ascending inside a group
    here; the kernel leaves that order open), counts[o] the ids for owner o and
    row_index each pair's position in send_ids (-1 when not requested)."""
    flat = np.asarray(ids, dtype=np.int64).reshape(-1)
    remote = (flat % world != rank) & ~np.isin(flat, np.asarray(ov_ids, dtype=np.int64))
    uniq = np.unique(flat[remote])
    send = uniq[np.argsort(uniq % world, kind="stable")]
    counts = np.bincount(send % world, minlength=world).astype(np.int64)
    order = np.argsort(send, kind="stable")
    rix = np.full(flat.shape, -1, dtype=np.int32)
    rix[remote] = order[np.searchsorted(send[order], flat[remote])]
    return send.astype(np.int32), counts, rix


def shard_route_push_ref(ids, ov_ids, world: int, rank: int):
    """The contract of engram_shard_route_push restated in numpy (a test
    reference): every (position, head) pair of `ids` ([n, n_heads]) whose owner
    id % world is another rank and which the overlay (ov_ids) does not serve
    sends its id to its owner; requests[o] lists owner o's ids in slot order
    (ascending pair index here; the kernel leaves the order open), counts[o]
    their number, and row_index each pair's row in the receive buffer (owners'
    blocks in ascending owner order: the counts of lower owners + its slot),
    -1 when not requested."""
    flat = np.asarray(ids, dtype=np.int64).reshape(-1)
    req = (flat % world != rank) & ~np.isin(flat, np.asarray(ov_ids, dtype=np.int64))
    owner = flat % world
    counts = np.bincount(owner[req], minlength=world).astype(np.int64)
    base = np.concatenate([[0], np.cumsum(counts)[:-1]])
    rix = np.full(flat.shape, -1, dtype=np.int64)
    requests = {}
    for o in range(world):
        sel = np.flatnonzero(req & (owner == o))
        requests[o] = flat[sel].astype(np.int32)
        rix[sel] = base[o] + np.arange(sel.size)
    return requests, counts, rix


def ple_block_torch(emb, hidden, w, hist, hc: int, n: int, eps: float, dil: int, detach_value: bool = False,
                    detach_gate: bool = False):
    """The PLE block's formula (engraft/replica/layers.py:565-626) restated in
    plain torch, differentiable, in the dtype of its inputs (the tests run it in
    float64 as the reference for the CUDA backward).  Returns (out, new_hist)."""
    import torch
    T = emb.shape[0]

    def rms(x, wt):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * wt.reshape(hc, n)

    key = (emb @ w["w_key"].T).reshape(T, hc, n)
    s = (rms(key, w["norm_key"]) * rms(hidden, w["norm_query"])).sum(-1) / n ** 0.5
    gate = torch.sigmoid(torch.sign(s) * torch.sqrt(s.abs().clamp(min=1e-6)))
    value = emb @ w["w_value"].T
    g = gate.detach() if detach_gate else gate
    v = value.detach() if detach_value else value
    gated = v.unsqueeze(1) * g.unsqueeze(-1)
    normed = rms(gated, w["norm_conv"])
    K = w["conv1d"].shape[1]
    H = hist.shape[0]
    full = torch.cat([hist, normed]).reshape(H + T, hc * n)
    pad = torch.cat([torch.zeros((K - 1) * dil, hc * n, dtype=full.dtype, device=full.device), full])
    acc = torch.zeros(T, hc * n, dtype=full.dtype, device=full.device)
    for k in range(K):
        back = (K - 1 - k) * dil
        # out t reads full row H + t - back, i.e. pad row (K-1)*dil + H + t - back; rows of pad before the
        # history are zeros, which is the reference's "no term before the history"
        lo = (K - 1) * dil + H - back
        acc = acc + pad[lo:lo + T] * w["conv1d"][:, k]
    out = hidden + gated + torch.nn.functional.silu(acc).reshape(T, hc, n)
    tail = (K - 1) * dil
    return out, torch.cat([hist, normed])[-tail:] if tail > 0 else normed[:0]
