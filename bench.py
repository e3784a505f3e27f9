#!/usr/bin/env python
"""Benchmark of the Engram/PLE table hot path on B200 (one JSON line on rank 0).

Default workload (BASELINE config 5 at N GPUs, weak scaling): per rank 64
sequences x 2048 tokens, Zipf(s=1.1) token ids over a 151,936-token vocabulary,
the full 320,001,536-row x 256 table in ggml IQ4_XS (resident, 46 GB), 40,000
fp32 overlay rows (the rows the batch reads most, as the descent's all-read
policy makes every read row variable), bigram+trigram pair sums added into a
bf16 residual stream [T, 2048].  One step = fused forward (hash -> overlay
probe -> gather/dequant -> residual add) + deterministic row-gradient backward
from a bf16 upstream gradient + the Adam step with the descent's regulariser.
With N > 1 ranks (weak scaling, each rank its own batch) the table is
row-sharded by default (owner = id mod N): each step's rows of other ranks are
routed three batches ahead, their ids stored straight into the owners' memory,
gathered there and copied back by the copy engines over NVLink.  The overlay
update crosses GPUs in peer memory: row gradients stored into their owners'
buffers by the backward, one Adam kernel per owner that stores the new rows
into every rank.  `--layout replicated` holds the whole table on every rank.

`--impl reference` times the CPU restatement of the reference's algorithm (the
oracle, all host threads) on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

VOCAB = 151_936
EOS = VOCAB - 1
FULL_ROWS = 320_001_536
METRIC = "Engram rows/s (fwd+bwd+Adam step, 64x2048-token Zipf batch per GPU, 320M-row x 256 IQ4_XS table)"
DEFAULT_STEPS, DEFAULT_WARMUP = 2000, 20

CONFIGS = {
    # name: (table rows, fmt, dim, sequences, seq_len, R, mode, backward)
    "cfg5": dict(rows=FULL_ROWS, fmt="iq4_xs", dim=256, seqs=64, seq_len=2048, R=40_000, mode="pairsum", bwd=True),
    "cfg2": dict(rows=FULL_ROWS, fmt="iq4_xs", dim=256, seqs=1, seq_len=2048, R=40_000, mode="pairsum", bwd=False),
    "cfg3": dict(rows=1 << 20, fmt="f32", dim=128, seqs=1, seq_len=2048, R=40_000, mode="concat", bwd=True),
    "cfg1": dict(rows=1 << 20, fmt="f32", dim=128, seqs=1, seq_len=2048, R=0, mode="concat", bwd=False),
    # decode-style: 256 sequences, 3 uniform history tokens + 1 new token; rows of the new tokens only
    "cfg4": dict(rows=1 << 20, fmt="f32", dim=128, seqs=256, seq_len=4, R=40_000, mode="concat", bwd=False,
                 decode=True),
}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=DEFAULT_STEPS)
    ap.add_argument("--warmup", type=int, default=DEFAULT_WARMUP)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--config", default="cfg5", choices=sorted(CONFIGS) + ["scan", "ple", "micro"])
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--projection", choices=["3xtf32", "tcgen05", "fp32"], default=None,
                    help="--config ple: the projections' engine (default: engraft_ngram_b200.ple.PROJECTION)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-latency", action="store_true",
                    help="N=1, config 5: skip the latency configurations (1, 2, 4 and the config-3 step)")
    ap.add_argument("--no-check", action="store_true",
                    help="skip the parity check of the timed kernels against the CPU oracle (N=1)")
    ap.add_argument("--table-rows", type=int, default=None, help="override (profiling a small case)")
    ap.add_argument("--seqs", type=int, default=None, help="override sequences per GPU")
    ap.add_argument("--exchange", choices=["peer", "nccl"], default="peer",
                    help="N>1, replicated table: the optimizer exchange as one peer-memory kernel per rank "
                         "(symmetric memory: engram_backward_to_owners + engram_adam_owner_step) or as NCCL reduce-scatter + all-gather")
    ap.add_argument("--shard-exchange", choices=["peer", "nccl"], default="peer",
                    help="--shard: rows read in place from their owners over NVLink (symmetric memory) or moved by "
                         "NCCL all-to-all of ids and rows")
    ap.add_argument("--e2e-exchange", choices=["nccl", "peer"], default="peer",
                    help="N>1 e2e through autograd: NCCL all-reduce of rows_var.grad + OverlayAdam, or the row "
                         "gradients stored into their owners (PeerRows.attach) + PeerAdam")
    ap.add_argument("--no-sharded-line", action="store_true",
                    help="N>1: skip the second measurement with the table row-sharded")
    ap.add_argument("--layout", choices=["sharded", "replicated"], default="sharded",
                    help="N>1, config 5: the table row-sharded across the ranks (owner = id mod N; each rank's "
                         "remote rows routed three batches ahead, gathered by their owners and copied with the copy "
                         "engines over NVLink), or replicated on every rank; the other layout is measured beside it")
    ap.add_argument("--stage", choices=["exchange", "push", "pull", "off"], default="exchange",
                    help="--shard, peer reads: copy the next step's rows of other ranks on a side stream while the "
                         "current step runs (ShardedTable.prefetch), so the forward reads every row locally; push: "
                         "the owners store them into the requesters' stages; pull: each rank loads its own")
    ap.add_argument("--stage-blocks", type=int, default=0,
                    help="grid cap of the staging copy (0: the whole GPU)")
    ap.add_argument("--shard", action="store_true",
                    help="row-sharded table: each rank holds rows g with g %% N == rank; rows move by NCCL all-to-all")
    return ap.parse_args()


def measured_peak_gbs():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return 6650.0, "fallback"


def profiled_traffic(kernel_tag: str):
    """dram bytes per launch of the forward kernel from the committed ncu summary."""
    for f in sorted((ROOT / "profiles").glob("*.md")):
        m = re.search(rf"{kernel_tag}.*?traffic_bytes_per_launch:\s*([0-9.eE+]+)", f.read_text(), flags=re.S)
        if m:
            return float(m.group(1)), f.name
    return None, None


# ---------------------------------------------------------------- workload
def zipf_cdf(torch, device, vocab=VOCAB, s=1.1):
    r = torch.arange(1, vocab + 1, dtype=torch.float64, device=device)
    c = torch.cumsum(r.pow(-s), 0)
    return c / c[-1]


def zipf_tokens(torch, n, gen, cdf):
    u = torch.rand(n, generator=gen, device=cdf.device, dtype=torch.float64)
    return torch.searchsorted(cdf, u).clamp_max(cdf.numel() - 1).to(torch.int32)


class Workload:
    """All inputs of one rank, resident on its GPU."""

    def __init__(self, cfg, rank, world, seed, device):
        import torch
        import engraft_ngram_b200 as eb
        from engraft_ngram_b200 import _lib as L
        from engraft_ngram_b200.table import synthetic_head_sizes, synthetic_multipliers, synthetic_resident
        self.cfg, self.rank, self.world, self.dev = cfg, rank, world, device
        self.L, self.eb = L, eb
        fmt = L.FMT_NAMES[cfg["fmt"]]
        self.fmt, self.dim = fmt, cfg["dim"]
        self.mode = L.MODE_PAIRSUM_ADD_BF16 if cfg["mode"] == "pairsum" else L.MODE_CONCAT_F32
        sizes = synthetic_head_sizes(cfg["rows"])
        offs = np.concatenate([[0], np.cumsum(sizes)[:-1]]).tolist()
        mult = synthetic_multipliers(seed)
        self.shard = None
        self.stage = False
        self.stage_blocks = int(cfg.get("stage_blocks", 0))
        if cfg.get("shard"):
            from engraft_ngram_b200.shard import ShardedTable, local_exchange, nccl_exchange, peer_shard_buffer
            n_local = (cfg["rows"] - rank + world - 1) // world
            if cfg.get("stage") == "exchange":
                # this rank's shard in plain local memory; the rows of other ranks arrive deduplicated through
                # owners' gathers and copy-engine transfers, staged three batches ahead
                # (ShardedTable.enable_exchange_staging)
                rows = synthetic_resident(n_local, fmt, self.dim, seed * 7919 + rank, device)
                self.shard = ShardedTable(rows, fmt, self.dim, sizes, offs, mult, EOS, world, rank, cfg["rows"])
                self.shard.enable_exchange_staging(cfg["seqs"] * cfg["seq_len"])
                self.exchange = None
                self.stage = "exchange"
            elif cfg.get("shard_exchange", "peer") == "peer" and world > 1:
                # every rank's shard in symmetric memory: the forward reads rows in place over NVLink
                buf, ptrs, self._shard_handle = peer_shard_buffer(cfg["rows"], fmt, self.dim, device)
                rows = synthetic_resident(n_local, fmt, self.dim, seed * 7919 + rank, device, out=buf)
                self.shard = ShardedTable(buf, fmt, self.dim, sizes, offs, mult, EOS, world, rank, cfg["rows"],
                                          peer_ptrs=ptrs)
                self.exchange = None
                self.stage = cfg.get("stage", "push") if cfg.get("stage", "push") in ("push", "pull") else False
                if self.stage == "push":
                    self.shard.enable_push_staging(cfg["seqs"] * cfg["seq_len"], max_blocks=self.stage_blocks)
            else:
                rows = synthetic_resident(n_local, fmt, self.dim, seed * 7919 + rank, device)
                self.shard = ShardedTable(rows, fmt, self.dim, sizes, offs, mult, EOS, world, rank, cfg["rows"])
                self.exchange = nccl_exchange() if world > 1 else local_exchange([self.shard])
                self.shard.exchange = self.exchange  # the public API (run_e2e) exchanges rows the same way
            self.table = self.shard
        else:
            rows = synthetic_resident(cfg["rows"], fmt, self.dim, seed, device)
            self.table = eb.DeviceTable(rows, fmt, self.dim, sizes, offs, mult, EOS, n_rows=cfg["rows"])
        self.decode = bool(cfg.get("decode"))
        self.T = cfg["seqs"] * cfg["seq_len"]
        cdf = zipf_cdf(torch, device)
        # the census batch (rank 0's) fixes the overlay rows identically on every rank
        gen0 = torch.Generator(device=device)
        gen0.manual_seed(seed * 1000 + 17)
        census = zipf_tokens(torch, self.T, gen0, cdf)
        gen = torch.Generator(device=device)
        gen.manual_seed(seed * 1000 + 17 + rank)
        self.tokens = census if rank == 0 else zipf_tokens(torch, self.T, gen, cdf)
        self.seg_start = (torch.arange(self.T, device=device, dtype=torch.int32) // cfg["seq_len"]) * cfg["seq_len"]
        # staged sharded reads: step k+1's rows are copied while step k runs; the two steps' batches live in two
        # buffers (same tokens here), so each copy is for a distinct batch
        # (the exchange is staged three batches ahead, so four batches are in flight: four buffers)
        self.depth = 3 if self.stage == "exchange" else 1
        self.tok_bufs = ([self.tokens] + [self.tokens.clone() for _ in range(self.depth)]) if self.stage else [self.tokens]
        self.tok_ready = torch.cuda.Event()  # the token buffers never change after this point
        self.tok_ready.record(torch.cuda.current_stream(device))
        self.k = 0
        self.positions = None
        if self.decode:  # uniform histories; output rows are the sequences' last tokens
            census = torch.randint(0, VOCAB, (self.T,), generator=gen0, device=device, dtype=torch.int32)
            self.tokens = census if rank == 0 else torch.randint(0, VOCAB, (self.T,), generator=gen, device=device,
                                                                 dtype=torch.int32)
            self.positions = torch.arange(cfg["seqs"], device=device, dtype=torch.int64) * cfg["seq_len"] + cfg["seq_len"] - 1
        R = cfg["R"]
        if R:
            ids = self.table.global_ids(census, self.seg_start)
            if self.decode:
                ids = ids[self.positions]
            ids = ids.reshape(-1).to(torch.int64)
            uniq, cnt = torch.unique(ids, return_counts=True)
            order = torch.argsort(cnt, descending=True, stable=True)  # ties -> smaller id first
            top = uniq[order[:R]]
            if top.numel() < R:  # pad with seeded rows never read, as the survey's config 3 does
                extra = torch.randint(0, cfg["rows"], (2 * R,), generator=gen0, device=device)
                extra = extra[~torch.isin(extra, uniq)]
                top = torch.cat([top, torch.unique(extra)[: R - top.numel()]])
            self.ov_ids = torch.sort(top).values.to(torch.int32)
        else:
            self.ov_ids = torch.zeros(0, dtype=torch.int32, device=device)
        self.R = int(self.ov_ids.numel())
        self.omap = eb.OverlayMap(self.ov_ids, device)
        self.remote_rows = 0  # row-sharded: (position, head) pairs per step served by other ranks (overlay heads skip)
        self.remote_distinct = 0  # ... and the distinct rows among them (what the exchange moves)
        if self.shard is not None and world > 1:
            ids = self.shard.global_ids(self.tokens, self.seg_start).reshape(-1)
            remote = (ids % world) != rank
            if self.R:
                remote &= ~torch.isin(ids, self.ov_ids)
            self.remote_rows = int(remote.sum())
            self.remote_distinct = int(torch.unique(ids[remote]).numel())
        if self.shard is not None:  # true rows live on their owners; start from seeded values instead
            gp = torch.Generator(device=device)
            gp.manual_seed(seed * 1000 + 5)
            self.p0 = torch.randn(self.R, self.dim, generator=gp, device=device) * 0.0085
        else:
            self.p0 = self.table.gather_rows(self.ov_ids) if self.R else torch.zeros(0, self.dim, device=device)
        self.peer = None
        if world > 1 and cfg.get("exchange", "peer") == "peer" and self.R and self.dim % 4 == 0:
            from engraft_ngram_b200.dist import PeerRows
            try:
                self.peer = PeerRows(self.R, self.dim, device)
            except Exception as exc:  # no symmetric memory here: keep the NCCL collectives, and say so
                print(f"[bench] peer-memory exchange unavailable ({exc!r}); using NCCL collectives", file=sys.stderr)
                cfg["exchange"] = "nccl"
        if self.peer is not None:
            self.peer.rows_var.copy_(self.p0)
            self.rows_var = self.peer.rows_var
            self.grad_rows = torch.zeros_like(self.p0)  # unused: the backward writes to the owners
        else:
            self.rows_var = self.p0.clone()
            self.grad_rows = torch.zeros_like(self.p0)
        nh, hpn = self.table.n_heads, 8
        self.nh, self.hpn = nh, hpn
        gg = torch.Generator(device=device)
        gg.manual_seed(seed * 1000 + 99 + rank)
        self.n_out = self.positions.numel() if self.decode else self.T
        if self.mode == L.MODE_PAIRSUM_ADD_BF16:
            self.out = (torch.randn(self.T, hpn * self.dim, generator=gg, device=device) * 0.5).to(torch.bfloat16)
            self.dout = (torch.randn(self.T, hpn * self.dim, generator=gg, device=device) * 1e-3).to(torch.bfloat16)
        else:
            self.out = torch.empty(self.n_out, nh, self.dim, device=device)
            self.dout = torch.randn(self.n_out, nh, self.dim, generator=gg, device=device) * 1e-3
        self.slots = torch.empty(self.n_out, nh, dtype=torch.int32, device=device)
        self.hits = torch.zeros(1, dtype=torch.int64, device=device)
        lib = L.load()
        self.ws_bytes = int(lib.engram_backward_workspace_bytes(self.T, nh, max(self.R, 1)))
        self.ws = torch.empty(self.ws_bytes, dtype=torch.uint8, device=device)
        from engraft_ngram_b200.dist import shard_bounds
        lo, hi = shard_bounds(self.R, world, rank)
        Rs = hi - lo
        self.Rs = Rs
        self.m = torch.zeros(max(Rs, 1), self.dim, device=device)
        self.v = torch.zeros(max(Rs, 1), self.dim, device=device)
        self.mu = 0.1
        from engraft_ngram_b200.optim import reg_scale
        self.reg_scale = reg_scale(self.mu, self.p0) if self.R else 0.0
        self.lr = 1e-3
        self.step_count = 0
        self.stream = torch.cuda.current_stream(device).cuda_stream
        self.ov_desc = self.omap.descriptor(self.rows_var) if self.R else L.EngramOverlay(None, 0, None, None, 0)

    def join_stage(self):
        """The current stream waits for the staging copy in flight (push: the
        copy and the barrier that completes it on every rank)."""
        import torch
        cur = torch.cuda.current_stream(self.dev)
        if self.shard.xstage is not None:
            cur.wait_stream(self.shard.xstage.side)
        elif self.shard.push is not None:
            self.shard.push.join(cur)
        elif self.shard._side is not None:
            cur.wait_stream(self.shard._side)

    # one step through the C ABI (device-resident inputs)
    def forward(self, hit_count=None):
        import ctypes as C
        if self.shard is not None:
            nb = len(self.tok_bufs)
            tok = self.tok_bufs[self.k % nb]
            if self.stage:  # a later step's rows of other ranks, staged while this step runs
                self.shard.prefetch(self.tok_bufs[(self.k + self.depth) % nb], self.seg_start,
                                    max_blocks=self.stage_blocks, omap=self.omap, ready=self.tok_ready)
            self.k += 1
            self.shard.forward(tok, self.seg_start, self.omap, self.rows_var, self.out, self.mode,
                               self.exchange, slots_out=self.slots if self.R else None, hit_count=hit_count)
            return
        if self.decode:
            st = self.L.load().engram_forward_at(C.byref(self.table.ctable), C.byref(self.ov_desc),
                                                 self.tokens.data_ptr(), self.T, self.seg_start.data_ptr(),
                                                 self.positions.data_ptr(), self.n_out, self.mode, self.out.data_ptr(),
                                                 None, self.slots.data_ptr() if self.R else None,
                                                 None if hit_count is None else hit_count.data_ptr(), self.stream)
            self.L.check(st, "engram_forward_at")
            return
        st = self.L.load().engram_forward(C.byref(self.table.ctable), C.byref(self.ov_desc), self.tokens.data_ptr(),
                                          self.seg_start.data_ptr(), 0, self.T, self.mode, self.out.data_ptr(), None,
                                          self.slots.data_ptr() if self.R else None,
                                          None if hit_count is None else hit_count.data_ptr(), self.stream)
        self.L.check(st, "engram_forward")

    def backward(self):
        if self.peer is not None:  # row gradients straight into their owners' receive buffers
            st = self.L.load().engram_backward_to_owners(self.slots.data_ptr(), self.T, self.nh, self.hpn, self.mode,
                                                         self.dout.data_ptr(), self.dim, self.R,
                                                         self.peer.recv_ptrs.data_ptr(), self.world, self.rank,
                                                         self.ws.data_ptr(), self.ws_bytes, self.stream)
            self.L.check(st, "engram_backward_to_owners")
            return
        st = self.L.load().engram_backward(self.slots.data_ptr(), self.T, self.nh, self.hpn, self.mode,
                                           self.dout.data_ptr(), self.dim, self.R, self.grad_rows.data_ptr(),
                                           self.ws.data_ptr(), self.ws_bytes, self.stream)
        self.L.check(st, "engram_backward")

    def optimizer(self, dist=None):
        """Adam (+ regulariser) on this rank's rows; with N ranks the row gradients
        are reduce-scattered first and the updated rows all-gathered after
        (engraft_ngram_b200.dist)."""
        from engraft_ngram_b200.dist import all_gather_rows, reduce_scatter_rows, shard_bounds
        self.step_count += 1
        lo, hi = shard_bounds(self.R, self.world, self.rank)
        if self.peer is not None:  # one kernel: sum over ranks, Adam, store into every rank's rows
            self.peer.step(self.m, self.v, self.p0[lo:hi], self.step_count, self.lr, 0.9, 0.999, 1e-8,
                           self.reg_scale)
            return
        p = self.rows_var[lo:hi]
        g = self.grad_rows[lo:hi] if dist is None else reduce_scatter_rows(self.grad_rows)
        st = self.L.load().engram_adam_step(p.data_ptr(), g.data_ptr(), self.m.data_ptr(), self.v.data_ptr(),
                                            self.p0[lo:hi].data_ptr(), p.numel(), self.step_count, self.lr,
                                            0.9, 0.999, 1e-8, self.reg_scale, self.stream)
        self.L.check(st, "engram_adam_step")
        if dist is not None:
            all_gather_rows(self.rows_var, p)

    def step(self, dist=None):
        self.forward()
        if self.cfg["bwd"]:
            if self.R:
                self.backward()
                self.optimizer(dist)

    def algorithmic_bytes(self):
        """Bytes the math must move once per step: the forward's token reads, the
        table rows of the non-overlay heads, the distinct overlay rows touched
        and the residual read + write (or the CONCAT output); the backward's dOut
        rows of the (position, group) pairs with a hit (of the hit heads in
        CONCAT mode) and the row-gradient writes; Adam's 8 floats per element of
        this rank's overlay rows."""
        import torch
        T, nh, hpn, dim = self.n_out, self.nh, self.hpn, self.dim
        raw_row = {self.L.FMT_F32: dim * 4, self.L.FMT_IQ4_NL: dim // 32 * 18, self.L.FMT_IQ4_XS: dim // 256 * 136}[self.fmt]
        self.hits.zero_()
        self.forward(self.hits)
        torch.cuda.synchronize()
        H = int(self.hits.item()) if self.R else 0
        slots = self.slots
        touched = int(torch.unique(slots[slots >= 0]).numel()) if self.R else 0
        fwd = 8 * T + raw_row * (nh * T - H) + 4 * dim * touched
        if self.mode == self.L.MODE_PAIRSUM_ADD_BF16:
            fwd += 2 * (T * hpn * dim * 2)
            pair_hit = ((slots[:, :hpn] >= 0) | (slots[:, hpn:] >= 0)).sum().item() if self.R else 0
            bwd = int(pair_hit) * dim * 2 + self.R * dim * 4
        else:
            fwd += T * nh * dim * 4
            bwd = H * dim * 4 + self.R * dim * 4
        adam = 8 * self.Rs * dim * 4
        if not self.cfg["bwd"] or not self.R:
            bwd = adam = 0
        return dict(fwd=fwd, bwd=bwd, adam=adam, hits=H, touched=touched)


# ------------------------------------------------------------ parity check
def parity_check(wl, n_sample=4096, seed=1234):
    """Checks the timed kernels on the full-size workload against the CPU
    oracle, outside the timed region, with the same C-ABI calls as the timed
    step (the oracle is the checker here, never the thing measured):
    - engram_hash ids and the timed forward's overlay slots, every (position,
      head) of the batch, against the oracle's hash (engraft/table.py:111-144)
      and row_map membership: bit-exact;
    - the bf16 residual of n_sample seeded positions after the timed forward,
      against the oracle's forward (IQ4_XS dequant engraft/replica/dequant.py:
      150-189, pair sums into the residual) run on those positions' rows, copied
      back from the resident table (every position reads heads whose global ids
      lie above 2^28, i.e. resident byte offsets above 2^32): bit-exact;
    - every overlay row gradient of the timed backward over the whole batch,
      against the oracle's in-order sums: bit-exact;
    - every row of one Adam step (engram_adam_step, with the descent's
      regulariser) from those gradients: bit-exact, and within 1e-5 of the
      row norm as the north star states.
    Returns the `parity` object of the bench line."""
    import ctypes as C
    import torch
    from oracle import oracle as O
    L, dev = wl.L, wl.dev
    lib = L.load()
    T, nh, hpn, dim, R = wl.T, wl.nh, wl.hpn, wl.dim, wl.R
    if wl.shard is not None or wl.decode or wl.fmt != L.FMT_IQ4_XS or wl.mode != L.MODE_PAIRSUM_ADD_BF16:
        return {"checked": False, "why": "the check covers the resident IQ4_XS pair-sum step"}
    t_begin = time.perf_counter()
    tab = wl.table
    gen = torch.Generator()
    gen.manual_seed(seed)
    sample = torch.sort(torch.randperm(T, generator=gen)[:n_sample]).values
    sample_dev = sample.to(dev)
    res_before = wl.out[sample_dev].view(torch.int16).cpu().numpy().view(np.uint16)
    ids_gpu = tab.global_ids(wl.tokens, wl.seg_start).cpu().numpy()
    hits = torch.zeros(1, dtype=torch.int64, device=dev)
    wl.forward(hits)  # the timed call: fused forward into the residual, slots out
    torch.cuda.synchronize()
    slots_gpu = wl.slots.cpu().numpy()
    res_after = wl.out[sample_dev].view(torch.int16).cpu().numpy().view(np.uint16)
    grad_gpu = torch.empty(R, dim, dtype=torch.float32, device=dev)
    st = lib.engram_backward(wl.slots.data_ptr(), T, nh, hpn, wl.mode, wl.dout.data_ptr(), dim, R,
                             grad_gpu.data_ptr(), wl.ws.data_ptr(), wl.ws_bytes, wl.stream)
    L.check(st, "engram_backward")
    p_gpu = wl.rows_var.detach().clone()
    m_gpu, v_gpu = torch.zeros_like(p_gpu), torch.zeros_like(p_gpu)
    st = lib.engram_adam_step(p_gpu.data_ptr(), grad_gpu.data_ptr(), m_gpu.data_ptr(), v_gpu.data_ptr(),
                              wl.p0.data_ptr(), p_gpu.numel(), 1, wl.lr, 0.9, 0.999, 1e-8, wl.reg_scale, wl.stream)
    L.check(st, "engram_adam_step")
    torch.cuda.synchronize()

    # the oracle on the host
    toks = wl.tokens.cpu().numpy()
    ss = wl.seg_start.cpu().numpy()
    ids_ref = O.hash_ids(toks, tab.ngram_size, tab.heads_per_ngram, tab.layer_multipliers, tab.head_vocab_sizes,
                         tab.head_offsets, tab.eos_token_id, seg_start=ss)
    ov_ids = wl.ov_ids.cpu().numpy()
    k = np.searchsorted(ov_ids, ids_ref)
    k_c = np.minimum(k, R - 1)
    slots_ref = np.where((k < R) & (ov_ids[k_c] == ids_ref), k_c, -1).astype(np.int32)
    # the sampled positions' rows, copied back from the resident table, as the reference's raw 136-byte rows
    s_ids = ids_ref[sample.numpy()]
    uniq, local = np.unique(s_ids, return_inverse=True)
    local = local.reshape(s_ids.shape).astype(np.int32)
    stride = tab.row_stride
    resident = tab.rows.view(tab.n_rows, stride)[torch.from_numpy(uniq.astype(np.int64)).to(dev)].cpu().numpy()
    raw = np.concatenate([resident[:, 128:136], resident[:, 0:128]], axis=1)  # [d|scales_h|scales_l][qs]
    pack_ok = bool(np.array_equal(O.pack(O.FMT_IQ4_XS, dim, raw), resident))
    pos_in = np.searchsorted(uniq, ov_ids)
    pos_c = np.minimum(pos_in, len(uniq) - 1)
    ov_local = np.where(uniq[pos_c] == ov_ids, pos_c, len(uniq) + np.arange(R)).astype(np.int32)
    rows_host = wl.rows_var.detach().cpu().numpy()
    out_ref, _ = O.forward(O.FMT_IQ4_XS, dim, raw, local, hpn, rows_host, ov_local, O.MODE_PAIRSUM_ADD_BF16,
                           residual=res_before)
    dout_host = wl.dout.view(torch.int16).cpu().numpy().view(np.uint16)
    g_ref = O.backward(slots_ref, hpn, dout_host, dim, R, O.MODE_PAIRSUM_ADD_BF16)
    p_ref, m_ref, v_ref = rows_host.copy(), np.zeros_like(rows_host), np.zeros_like(rows_host)
    O.adam_(p_ref, g_ref, m_ref, v_ref, 1, wl.lr, p0=wl.p0.cpu().numpy(), reg_scale=np.float32(wl.reg_scale))

    def diff(a, b):
        return int(np.count_nonzero(np.asarray(a).view(np.uint32 if np.asarray(a).itemsize == 4 else np.uint16)
                                    != np.asarray(b).view(np.uint32 if np.asarray(b).itemsize == 4 else np.uint16)))

    p_got = p_gpu.cpu().numpy()
    norm = np.linalg.norm(p_ref, axis=1, keepdims=True)
    rel = float((np.abs(p_got - p_ref) / np.maximum(norm, 1e-30)).max()) if R else 0.0
    read = slots_ref[sample.numpy()] < 0  # heads whose table row the forward dequantised
    big = s_ids >= (1 << 28)
    mism = {"ids": diff(ids_gpu, ids_ref), "slots": diff(slots_gpu, slots_ref),
            "residual": diff(res_after, out_ref), "row_gradients": diff(grad_gpu.cpu().numpy(), g_ref),
            "adam_rows": diff(p_got, p_ref), "adam_m": diff(m_gpu.cpu().numpy(), m_ref),
            "adam_v": diff(v_gpu.cpu().numpy(), v_ref), "resident_layout": 0 if pack_ok else 1}
    return {
        "checked": {"ids": int(ids_ref.size), "slots": int(slots_ref.size), "residual_values": int(out_ref.size),
                    "residual_positions": int(n_sample), "row_gradient_values": int(g_ref.size),
                    "adam_values": int(p_ref.size),
                    "table_rows_dequantised": int(read.sum()),
                    "table_rows_above_2^28": int((read & big).sum()),
                    "max_resident_byte_offset": int(int(s_ids[read].max()) * stride) if read.any() else 0},
        "mismatches": mism, "all_bit_exact": not any(mism.values()),
        "adam_max_abs_err_rel_row_norm": rel, "tolerance_rel_row_norm": 1e-5, "within_tolerance": rel <= 1e-5,
        "oracle": "oracle/engram_oracle.c (C restatement of the reference path), host threads", "seconds":
            round(time.perf_counter() - t_begin, 2)}


# ------------------------------------------------------------------ clocks
class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        import torch
        try:
            self.idx = "GPU-" + str(torch.cuda.get_device_properties(gpu_index).uuid)
        except Exception:
            self.idx = str(gpu_index)
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        self.samples = []
        if self.proc is None:
            return
        time.sleep(0.15)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out = ""
        for line in out.splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                self.samples.append(parts)

    def summary(self):
        s = getattr(self, "samples", [])
        if not s:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        def num(x):
            try:
                return float(x)
            except ValueError:
                return None
        sm = [num(x[1]) for x in s if num(x[1]) is not None]
        power = [num(x[3]) for x in s if num(x[3]) is not None]
        load = [v for v, p in zip(sm, power) if p is not None and p > 250] or sm
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[k] for x in s for k in range(4) if x[5 + k].lower().startswith("active")})
        return {"sm_mhz": statistics.median(load) if load else None, "sm_max_mhz": num(s[0][2]),
                "reasons": reasons, "samples": len(s), "power_w_max": max(power) if power else None}


# ------------------------------------------------------------- CPU oracle
def cpu_oracle_step_time(cfg, seed, budget_s=10.0):
    """Times the oracle (CPU restatement of the reference path, all host
    threads) on a bounded sample and extrapolates to one full step.
    Table: a 2^24-row slice of the same format (host RAM), head sizes scaled."""
    from oracle import oracle as O
    from engraft_ngram_b200.table import synthetic_head_sizes, synthetic_multipliers
    fmt = {"f32": O.FMT_F32, "iq4_nl": O.FMT_IQ4_NL, "iq4_xs": O.FMT_IQ4_XS}[cfg["fmt"]]
    dim = cfg["dim"]
    n_rows = min(cfg["rows"], 1 << 22)
    rb = O.raw_row_bytes(fmt, dim)
    rng = np.random.default_rng(seed)
    raw = np.frombuffer(rng.bytes(n_rows * rb), dtype=np.uint8).reshape(n_rows, rb).copy()
    if fmt == O.FMT_F32:
        raw = (rng.standard_normal((n_rows, dim)) * 0.0085).astype(np.float32).view(np.uint8).reshape(n_rows, rb)
    else:
        nb = dim // (256 if fmt == O.FMT_IQ4_XS else 32)
        bs = 136 if fmt == O.FMT_IQ4_XS else 18
        d = np.abs(rng.standard_normal((n_rows, nb)) * 1e-3).astype(np.float16)
        raw.reshape(n_rows, nb, bs)[:, :, 0:2] = d.view(np.uint8).reshape(n_rows, nb, 2)
    sizes = synthetic_head_sizes(n_rows)
    offs = np.concatenate([[0], np.cumsum(sizes)[:-1]]).tolist()
    mult = synthetic_multipliers(seed)
    T_full = cfg["seqs"] * cfg["seq_len"]
    T_s = min(T_full, 8192)
    ranks = np.arange(1, VOCAB + 1, dtype=np.float64)
    cdf = np.cumsum(ranks ** -1.1)
    cdf /= cdf[-1]
    toks = np.searchsorted(cdf, rng.random(T_s)).astype(np.int32)
    ss = ((np.arange(T_s) // cfg["seq_len"]) * cfg["seq_len"]).astype(np.int32)
    hpn, dimr = 8, dim
    R = cfg["R"]
    ids0 = O.hash_ids(toks, 3, 8, mult, sizes, offs, EOS, seg_start=ss)
    u, c = np.unique(ids0, return_counts=True)
    ov = np.sort(u[np.argsort(-c, kind="stable")][:R]).astype(np.int32) if R else np.zeros(0, np.int32)
    Rr = len(ov)
    rows0 = O.dequant(fmt, dim, raw[ov]) if Rr else np.zeros((0, dim), np.float32)
    pairsum = cfg["mode"] == "pairsum"
    res = O.bf16_bits(rng.standard_normal((T_s, hpn * dimr)).astype(np.float32) * 0.5) if pairsum else None
    dout = (O.bf16_bits(rng.standard_normal((T_s, hpn * dimr)).astype(np.float32) * 1e-3) if pairsum
            else (rng.standard_normal((T_s, 16, dimr)) * 1e-3).astype(np.float32))
    p = rows0.copy()
    m = np.zeros_like(p)
    v = np.zeros_like(p)
    rs = O.reg_scale(0.1, rows0) if Rr else 0.0
    mode = O.MODE_PAIRSUM_ADD_BF16 if pairsum else O.MODE_CONCAT_F32

    def fwd_bwd():
        ids = O.hash_ids(toks, 3, 8, mult, sizes, offs, EOS, seg_start=ss)
        _, slots = O.forward(fmt, dim, raw, ids, 8, p, ov, mode, residual=res)
        if cfg["bwd"] and Rr:
            O.backward(slots, 8, dout, dim, Rr, mode)

    def adam(nrows):
        if cfg["bwd"] and Rr:
            O.adam_(p[:nrows], np.zeros((nrows, dim), np.float32), m[:nrows], v[:nrows], 1, 1e-3, p0=rows0[:nrows],
                    reg_scale=rs)

    # repeat the sample until about budget_s seconds of CPU work, then take medians
    t_fbs, t_adams = [], []
    t_begin = time.perf_counter()
    while True:
        t0 = time.perf_counter()
        fwd_bwd()
        t_fbs.append(time.perf_counter() - t0)
        t0 = time.perf_counter()
        adam(Rr)
        t_adams.append(time.perf_counter() - t0)
        if time.perf_counter() - t_begin >= budget_s:
            break
    t_fb, t_adam = statistics.median(t_fbs), statistics.median(t_adams)
    t_step = t_fb * (T_full / T_s) + t_adam * (cfg["R"] / max(Rr, 1))
    return dict(t_step=t_step, t_fb=t_fb, t_adam=t_adam, T_s=T_s, T_full=T_full, R=Rr, n_rows=n_rows,
                threads=O.num_threads(), fwd_bwd=fwd_bwd, adam=adam, repeats=len(t_fbs),
                cpu_seconds=time.perf_counter() - t_begin)


def run_reference(args, cfg, rank):
    """--impl reference: the oracle port on the host cores, bounded samples per step."""
    if rank != 0:
        return
    cores = os.cpu_count()
    base = cpu_oracle_step_time(cfg, args.seed)
    T_full = base["T_full"]
    # per-step sample: a fraction of the positions and of the Adam rows so the
    # whole run ends within a few minutes
    per_step_budget = max(0.02, 150.0 / max(1, args.steps + args.warmup))
    frac = min(1.0, per_step_budget / max(base["t_step"], 1e-9))
    T_s = base["T_s"]
    # each step runs the whole sample batch (T_s positions: the unit the oracle call takes) and scales its
    # time by T_full / T_s; the Adam sample is the fraction `frac` of the overlay rows, scaled by R / rows
    scale_fb = T_full / T_s
    times = []
    for k in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        base["fwd_bwd"]()
        t_fb = time.perf_counter() - t0
        t1 = time.perf_counter()
        nrows = max(1, int(base["R"] * min(1.0, frac)))
        base["adam"](nrows)
        t_ad = time.perf_counter() - t1
        if k >= args.warmup:
            times.append(t_fb * scale_fb + t_ad * (cfg["R"] / nrows if base["R"] else 0))
        if time.perf_counter() - START > 170:
            break
    t_step = statistics.median(times) if times else base["t_step"]
    value = 16 * T_full / t_step
    line = {
        "metric": METRIC, "value": value, "unit": "rows/s", "impl": "reference", "n_gpus": args.gpus,
        "steps": len(times), "warmup": args.warmup, "ms_per_step": t_step * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_json(cfg, args),
        "cpu_baseline": {"value": value, "unit": "rows/s", "cores": base["threads"], "kind": "port",
                         "sample": f"oracle (C restatement, OpenMP {base['threads']} threads of {cores}) on "
                                   f"{base['T_s']} positions x 16 rows per step, time x{scale_fb:.0f} (extrapolated "
                                   f"to {T_full} positions), Adam over {max(1, int(base['R'] * frac))} of the overlay "
                                   f"rows, time scaled to R={cfg['R']}; table slice {base['n_rows']} rows"},
        "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_latency(wl, args, device):
    """The latency configurations of BASELINE on one GPU, measured after the
    headline step (CUDA events on the launching stream, inputs resident):
    - cfg2: 1 x 2048 Zipf tokens, forward only, pair sums into a bf16 [2048,
      2048] residual, on the resident 320M-row IQ4_XS table (no overlay);
    - cfg1: 1 x 2048 uniform tokens, forward only, CONCAT fp32 [2048, 16, 128],
      on a 2^20 x 128 fp32 table (no overlay);
    - cfg4: 256 sequences x 1 new token (3 uniform history tokens each), CONCAT,
      on the cfg1 table with 40,000 overlay rows (engram_forward_at);
    - cfg3: the training step on the cfg1 table (2048 Zipf tokens, 40,000
      overlay rows, CONCAT): forward, row gradients, Adam with the regulariser.
    Each runs over 64 distinct batches (inputs and outputs larger than L2):
    once as 64 separate launches ("stream"), once as the 64 calls captured in
    one CUDA graph and replayed ("graph"); us per call, rows/s and algorithmic
    GB/s of the graph replay."""
    import ctypes as C
    import torch
    import engraft_ngram_b200 as eb
    from engraft_ngram_b200 import _lib as L
    from engraft_ngram_b200.table import synthetic_head_sizes, synthetic_multipliers, synthetic_resident
    lib = L.load()
    B = 64
    out = {}
    cdf = zipf_cdf(torch, device)
    gen = torch.Generator(device=device)
    gen.manual_seed(args.seed * 1000 + 31)

    def measure(calls, rows_per_call, bytes_per_call):
        """calls: list of B zero-argument launches on the current stream."""
        stream = torch.cuda.current_stream(device)
        for c in calls[:3]:
            c()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for c in calls:
            c()
        e1.record()
        torch.cuda.synchronize()
        t_stream = e0.elapsed_time(e1) / len(calls)
        g = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(device)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            for c in calls[:2]:
                c()
        stream.wait_stream(side)
        torch.cuda.synchronize()
        with torch.cuda.graph(g):
            for c in calls:
                c()
        g.replay()
        torch.cuda.synchronize()
        reps = 5
        e0.record()
        for _ in range(reps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        t_graph = e0.elapsed_time(e1) / (reps * len(calls))
        del g
        return {"us_per_call_stream": t_stream * 1e3, "us_per_call_graph": t_graph * 1e3,
                "rows_per_s_graph": rows_per_call / (t_graph * 1e-3),
                "gbps_graph": bytes_per_call / (t_graph * 1e-3) / 1e9, "algorithmic_bytes_per_call": bytes_per_call}

    ov0 = L.EngramOverlay(None, 0, None, None, 0)
    T = 2048
    # cfg2 on the headline table
    if wl.shard is None and wl.fmt == L.FMT_IQ4_XS and wl.dim == 256:
        toks = [zipf_tokens(torch, T, gen, cdf) for _ in range(B)]
        res = (torch.randn(B, T, 8 * 256, generator=gen, device=device) * 0.5).to(torch.bfloat16)
        ct = wl.table.ctable

        def f2(k):
            return lambda: L.check(lib.engram_forward(C.byref(ct), C.byref(ov0), toks[k].data_ptr(), None, 0, T,
                                                      L.MODE_PAIRSUM_ADD_BF16, res[k].data_ptr(), None, None, None,
                                                      torch.cuda.current_stream(device).cuda_stream), "engram_forward")
        out["cfg2"] = measure([f2(k) for k in range(B)], 16 * T, T * (4 + 16 * 136 + 2 * 2 * 8 * 256))
        out["cfg2"]["workload"] = "1x2048 Zipf tokens, 320M-row x 256 IQ4_XS table, pair sums into bf16 [2048, 2048]"
        del res, toks
    # the cfg1 table
    n1, dim = 1 << 20, 128
    sizes = synthetic_head_sizes(n1)
    offs = np.concatenate([[0], np.cumsum(sizes)[:-1]]).tolist()
    t1 = eb.DeviceTable(synthetic_resident(n1, L.FMT_F32, dim, args.seed + 1, device), L.FMT_F32, dim, sizes, offs,
                        synthetic_multipliers(args.seed), EOS, n_rows=n1)
    ct1 = t1.ctable
    utoks = [torch.randint(0, VOCAB, (T,), generator=gen, device=device, dtype=torch.int32) for _ in range(B)]
    emb = torch.empty(B, T, 16, dim, device=device)

    def f1(k):
        return lambda: L.check(lib.engram_forward(C.byref(ct1), C.byref(ov0), utoks[k].data_ptr(), None, 0, T,
                                                  L.MODE_CONCAT_F32, emb[k].data_ptr(), None, None, None,
                                                  torch.cuda.current_stream(device).cuda_stream), "engram_forward")
    out["cfg1"] = measure([f1(k) for k in range(B)], 16 * T, T * (4 + 2 * 16 * dim * 4))
    out["cfg1"]["workload"] = "1x2048 uniform tokens, 2^20 x 128 fp32 table, CONCAT fp32 [2048, 16, 128]"
    del emb, utoks
    # overlay of the cfg1 table: the 40,000 rows a Zipf census batch reads most
    R = 40_000
    census = zipf_tokens(torch, T * 16, gen, cdf)
    ids = t1.global_ids(census).reshape(-1).to(torch.int64)
    uniq, cnt = torch.unique(ids, return_counts=True)
    top = uniq[torch.argsort(cnt, descending=True, stable=True)[:R]]
    if top.numel() < R:
        extra = torch.randint(0, n1, (4 * R,), generator=gen, device=device)
        top = torch.cat([top, torch.unique(extra[~torch.isin(extra, uniq)])[: R - top.numel()]])
    ov_ids = torch.sort(top).values.to(torch.int32)
    omap = eb.OverlayMap(ov_ids, device)
    p0 = t1.gather_rows(ov_ids)
    rows_var = p0.clone()
    ovd = omap.descriptor(rows_var)
    # cfg4: decode-style
    S, H = 256, 4
    dtoks = [torch.randint(0, VOCAB, (S * H,), generator=gen, device=device, dtype=torch.int32) for _ in range(B)]
    seg = (torch.arange(S * H, device=device, dtype=torch.int32) // H) * H
    pos = torch.arange(S, device=device, dtype=torch.int64) * H + H - 1
    demb = torch.empty(B, S, 16, dim, device=device)

    def f4(k):
        return lambda: L.check(lib.engram_forward_at(C.byref(ct1), C.byref(ovd), dtoks[k].data_ptr(), S * H,
                                                     seg.data_ptr(), pos.data_ptr(), S, L.MODE_CONCAT_F32,
                                                     demb[k].data_ptr(), None, None, None,
                                                     torch.cuda.current_stream(device).cuda_stream), "engram_forward_at")
    out["cfg4"] = measure([f4(k) for k in range(B)], 16 * S, S * (3 * 4 + 2 * 16 * dim * 4))
    out["cfg4"]["workload"] = "256 sequences x 1 new token (3 uniform history tokens), cfg1 table, 40,000 overlay rows"
    del demb, dtoks
    # cfg3: the training step on the cfg1 table
    ztoks = [zipf_tokens(torch, T, gen, cdf) for _ in range(B)]
    cemb = torch.empty(T, 16, dim, device=device)
    slots = torch.empty(T, 16, dtype=torch.int32, device=device)
    dout = torch.randn(B, T, 16, dim, generator=gen, device=device) * 1e-3
    grad = torch.empty(R, dim, device=device)
    m, v = torch.zeros(R, dim, device=device), torch.zeros(R, dim, device=device)
    wsb = int(lib.engram_backward_workspace_bytes(T, 16, R))
    ws = torch.empty(wsb, dtype=torch.uint8, device=device)
    from engraft_ngram_b200.optim import reg_scale
    rs = reg_scale(0.1, p0)

    def f3(k):
        def step():
            s = torch.cuda.current_stream(device).cuda_stream
            L.check(lib.engram_forward(C.byref(ct1), C.byref(ovd), ztoks[k].data_ptr(), None, 0, T, L.MODE_CONCAT_F32,
                                       cemb.data_ptr(), None, slots.data_ptr(), None, s), "engram_forward")
            L.check(lib.engram_backward(slots.data_ptr(), T, 16, 8, L.MODE_CONCAT_F32, dout[k].data_ptr(), dim, R,
                                        grad.data_ptr(), ws.data_ptr(), wsb, s), "engram_backward")
            L.check(lib.engram_adam_step(rows_var.data_ptr(), grad.data_ptr(), m.data_ptr(), v.data_ptr(),
                                         p0.data_ptr(), rows_var.numel(), 1, 1e-3, 0.9, 0.999, 1e-8, rs, s),
                    "engram_adam_step")
        return step
    step_bytes = T * (4 + 2 * 16 * dim * 4 + 16 * dim * 4) + 9 * R * dim * 4
    out["cfg3"] = measure([f3(k) for k in range(B)], 16 * T, step_bytes)
    out["cfg3"]["workload"] = ("training step: 2048 Zipf tokens, cfg1 table, 40,000 overlay rows, forward + row "
                               "gradients + Adam (the Adam step count is held at 1 in the replayed graph)")
    del dout, cemb
    out["cfg3_dropin"] = run_dropin(t1, ov_ids, p0, ztoks, device, args)
    # the reference's own format: 160-wide IQ4_NL rows
    n_nl = 1 << 20
    t_nl = eb.DeviceTable(synthetic_resident(n_nl, L.FMT_IQ4_NL, 160, args.seed + 2, device), L.FMT_IQ4_NL, 160,
                          sizes, offs, synthetic_multipliers(args.seed), EOS, n_rows=n_nl)
    out["cfg3_dropin_iq4nl160"] = run_dropin(t_nl, ov_ids, t_nl.gather_rows(ov_ids), ztoks, device, args)
    return out


def run_dropin(table, ov_ids, p0, toks, device, args, K=40):
    """The reference's own call path through the drop-in: each step builds
    OverlayEmb(table, tokens as a Python list, rows_var, row_map as a dict)
    .build(2048) (engraft/replica/seq.py:1430-1432), backpropagates a gradient
    and steps OverlayAdam with the descent's regulariser
    (engraft/descend_corpus.py:921-947).  Reports the wall time per step
    (synchronised at the end of K steps), the host (Python) time per step and
    the device time (CUDA events around the K steps)."""
    import torch
    import engraft_ngram_b200 as eb
    T = 2048
    R = int(ov_ids.numel())
    row_map = {int(g): k for k, g in enumerate(ov_ids.cpu().tolist())}
    tok_lists = [t.cpu().tolist() for t in toks[:8]]
    rows_var = p0.clone().requires_grad_(True)
    opt = eb.OverlayAdam([rows_var], lr=1e-3, reg_ref=p0, reg_mu=0.1)
    g = torch.Generator(device=device)
    g.manual_seed(args.seed * 1000 + 77)
    douts = [torch.randn(T, 16 * table.dim, generator=g, device=device) * 1e-3 for _ in range(4)]
    hits = []

    def step(k):
        opt.zero_grad()
        ov = eb.OverlayEmb(table, tok_lists[k % len(tok_lists)], rows_var, row_map)
        emb = ov.build(T)
        emb.backward(douts[k % len(douts)])
        opt.step()
        return ov

    for k in range(3):
        step(k)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    host = 0.0
    t0 = time.perf_counter()
    e0.record()
    last = None
    for k in range(K):
        h0 = time.perf_counter()
        last = step(k)
        host += time.perf_counter() - h0
    e1.record()
    torch.cuda.synchronize()
    wall = (time.perf_counter() - t0) / K
    dev_ms = e0.elapsed_time(e1) / K
    hits = last.n_id_hits
    return {"us_per_step_wall": wall * 1e6, "host_us_per_step": host / K * 1e6, "device_us_per_step": dev_ms * 1e3,
            "host_fraction": (host / K) / wall, "rows_per_s": 16 * T / wall, "n_id_hits_last": int(hits),
            "api": "OverlayEmb(table, tokens list, rows_var, row_map dict).build(2048) + backward + OverlayAdam.step",
            "workload": f"2048 Zipf tokens, {table.n_rows}-row x {table.dim} table (fmt {table.fmt}), R={R}"}


def run_scan(args, device):
    """Throughput of the bulk hash + overlay hit scan (engraft/damage.py:168-224) on
    a device-resident Zipf corpus: positions/s (16 rows each)."""
    import ctypes as C
    import torch
    import engraft_ngram_b200 as eb
    from engraft_ngram_b200 import _lib as L
    from engraft_ngram_b200.table import synthetic_head_sizes, synthetic_multipliers
    n = 64 * 1024 * 1024
    sizes = synthetic_head_sizes(FULL_ROWS)
    offs = np.concatenate([[0], np.cumsum(sizes)[:-1]]).tolist()
    dt = eb.DeviceTable(torch.zeros(64, dtype=torch.uint8, device=device), L.FMT_F32, 4, sizes, offs,
                        synthetic_multipliers(args.seed), EOS, n_rows=FULL_ROWS, hash_only=True)
    g = torch.Generator(device=device)
    g.manual_seed(args.seed)
    toks = zipf_tokens(torch, n, g, zipf_cdf(torch, device))
    ids = dt.global_ids(toks[: 1 << 20]).reshape(-1)
    ov = torch.unique(ids)[::7][:14_032].to(torch.int32)  # s0b-sized overlay of rows the corpus reads
    R = ov.numel()
    omap = eb.OverlayMap(ov, device)
    ovd = L.EngramOverlay(None, R, omap.keys.data_ptr(), omap.slots.data_ptr(), omap.capacity)
    dnorm = torch.rand(R, generator=g, device=device) * 0.2
    lib = L.load()
    wsb = int(lib.engram_scan_hits_workspace_bytes(n))
    ws = torch.empty(wsb, dtype=torch.uint8, device=device)
    pos = torch.empty(n, dtype=torch.int64, device=device)
    nh = torch.empty(n, dtype=torch.int32, device=device)
    dmax = torch.empty(n, dtype=torch.float32, device=device)
    dsum = torch.empty(n, dtype=torch.float32, device=device)
    nhits = torch.zeros(1, dtype=torch.int64, device=device)
    rc = torch.zeros(R, dtype=torch.int64, device=device)
    stream = torch.cuda.current_stream(device).cuda_stream

    def once():
        st = lib.engram_scan_hits(C.byref(dt.ctable), toks.data_ptr(), 0, n, 0, 1, C.byref(ovd), dnorm.data_ptr(),
                                  pos.data_ptr(), nh.data_ptr(), dmax.data_ptr(), dsum.data_ptr(), nhits.data_ptr(),
                                  rc.data_ptr(), ws.data_ptr(), wsb, stream)
        L.check(st, "engram_scan_hits")

    for _ in range(3):
        once()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    K = max(1, min(args.steps, 50))
    e0.record()
    for _ in range(K):
        once()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / K
    line = {"metric": "overlay hit scan positions/s (damage.scan_hits, 64M-token Zipf corpus, 320M-row table)",
            "value": n / (ms * 1e-3), "unit": "positions/s", "ms_per_scan": ms, "n_hits": int(nhits.item()),
            "overlay_rows": R, "config": {"workload": "scan: 67,108,864 tokens resident, 16 rows each"}}
    print(json.dumps(line), flush=True)


def run_ple(args, device):
    """The PLE block after the gather (engraft/replica/layers.py:565-626) at the
    reference's width (hc = 4, n_embd = 2560, 4 conv taps, dilation 3) over
    2048 positions: the two fp32 projection GEMMs (cuBLAS) and the two block
    kernels, each timed with CUDA events; positions/s for the whole block."""
    import types
    import torch
    import engraft_ngram_b200 as eb
    from engraft_ngram_b200 import _lib as L
    hc, n, K, dil, T = 4, 2560, 4, 3, 2048
    g = torch.Generator(device=device)
    g.manual_seed(args.seed)
    r = lambda *s: torch.randn(*s, generator=g, device=device) * 0.1  # noqa: E731
    w = types.SimpleNamespace(w_key=r(hc * n, n), w_value=r(n, n), norm_key=1 + r(hc * n), norm_query=1 + r(hc * n),
                              norm_conv=1 + r(hc * n), conv1d=r(hc * n, K))
    emb, hidden, hist = r(T, n), r(T, hc, n), r((K - 1) * dil, hc, n)
    hp = types.SimpleNamespace(hc_mult=hc, n_embd=n, f_norm_rms_eps=1e-6, ple_ngram_size=dil)
    lib = L.load()
    stream = torch.cuda.current_stream(device).cuda_stream
    from engraft_ngram_b200 import ple as P
    if args.projection:
        P.PROJECTION = args.projection
    kv = torch.empty(T, hc * n + n, device=device)
    value = kv[:, hc * n:]
    gate, normed, out = (torch.empty(T, hc, device=device), torch.empty(T, hc, n, device=device),
                         torch.empty(T, hc, n, device=device))
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    K_steps = max(1, min(args.steps, 50))
    for _ in range(3):
        eb.ple_forward(emb, hidden, w, hist, hp)
    torch.cuda.synchronize()
    stride = hc * n + n
    t_fp32 = 0.0
    for _ in range(K_steps):  # the plain fp32 projection, for comparison
        ev[0].record()
        P.project(emb, w, kv, "fp32")
        ev[1].record()
        torch.cuda.synchronize()
        t_fp32 += ev[0].elapsed_time(ev[1])
    t_gemm = t_gate = t_conv = 0.0
    for _ in range(K_steps):  # the same launches as ple_forward, with events between them
        ev[0].record()
        P.project(emb, w, kv)
        ev[1].record()
        L.check(lib.engram_ple_gate(kv.data_ptr(), stride, value.data_ptr(), stride, hidden.data_ptr(),
                                    w.norm_key.data_ptr(), w.norm_query.data_ptr(), w.norm_conv.data_ptr(), T, hc, n,
                                    1e-6, gate.data_ptr(), None, normed.data_ptr(), stream), "engram_ple_gate")
        ev[2].record()
        L.check(lib.engram_ple_conv(value.data_ptr(), stride, hidden.data_ptr(), gate.data_ptr(), normed.data_ptr(),
                                    hist.data_ptr(), hist.shape[0], w.conv1d.data_ptr(), K, dil, T, hc, n,
                                    out.data_ptr(), stream), "engram_ple_conv")
        ev[3].record()
        torch.cuda.synchronize()
        t_gemm += ev[0].elapsed_time(ev[1])
        t_gate += ev[1].elapsed_time(ev[2])
        t_conv += ev[2].elapsed_time(ev[3])
    t_gemm, t_gate, t_conv, t_fp32 = (x / K_steps for x in (t_gemm, t_gate, t_conv, t_fp32))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(K_steps):
        eb.ple_forward(emb, hidden, w, hist, hp)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / K_steps
    peak, peak_kind = measured_peak_gbs()
    C = T * hc * n * 4
    gate_bytes = 2 * C + T * n * 4 + C + 3 * hc * n * 4  # key, hidden, value, normed out, norm weights
    conv_bytes = C + C + T * n * 4 + C + hc * n * K * 4  # normed, hidden, value, out, conv weights
    flops = 2.0 * T * n * (hc * n + n)
    line = {"metric": "PLE block positions/s (layers.ple_forward, hc=4, n_embd=2560, 2048 positions, fp32)",
            "value": T / (ms * 1e-3), "unit": "positions/s", "ms_per_call": ms,
            "phase_ms": {f"projections_{P.PROJECTION}": t_gemm, "engram_ple_gate": t_gate, "engram_ple_conv": t_conv},
            "gemm_tflops": flops / (t_gemm * 1e-3) / 1e12,
            "projections_fp32_sgemm": {"ms": t_fp32, "tflops": flops / (t_fp32 * 1e-3) / 1e12},
            "roofline": {"engram_ple_gate": {"bound": "hbm", "achieved": gate_bytes / (t_gate * 1e-3) / 1e9,
                                             "peak": peak, "unit": "GB/s", "frac": gate_bytes / (t_gate * 1e-3) / 1e9 / peak},
                         "engram_ple_conv": {"bound": "hbm", "achieved": conv_bytes / (t_conv * 1e-3) / 1e9,
                                             "peak": peak, "unit": "GB/s", "frac": conv_bytes / (t_conv * 1e-3) / 1e9 / peak},
                         "peak_source": peak_kind},
            "config": {"workload": "ple: 2048 positions, hc=4, n_embd=2560, K=4, dilation 3, history 9 rows"}}
    print(json.dumps(line), flush=True)


def run_micro(args, device):
    """The kernels off the config-5 step, each on a workload of its own at the
    headline table's size, timed with CUDA events over K launches after three
    warm-up launches: achieved GB/s = the bytes the call must move (stated per
    kernel) / its mean time, against the measured copy peak.  One JSON line.
    Also the command the per-kernel ncu summaries are captured from
    (--table-rows shrinks the table and the hashed stream for multi-pass
    captures)."""
    import ctypes as C
    import torch
    import engraft_ngram_b200 as eb
    from engraft_ngram_b200 import _lib as L
    from engraft_ngram_b200.table import synthetic_head_sizes, synthetic_multipliers
    lib = L.load()
    stream = torch.cuda.current_stream(device).cuda_stream
    peak, peak_kind = measured_peak_gbs()
    K = max(1, min(args.steps, 50))
    g = torch.Generator(device=device)
    g.manual_seed(args.seed)
    cdf = zipf_cdf(torch, device)
    n_rows = args.table_rows or FULL_ROWS
    sizes = synthetic_head_sizes(n_rows)
    offs = np.concatenate([[0], np.cumsum(sizes)[:-1]]).tolist()
    mult = synthetic_multipliers(args.seed)
    fmt, dim = L.FMT_IQ4_XS, 256
    addr = eb.DeviceTable(torch.zeros(64, dtype=torch.uint8, device=device), fmt, dim, sizes, offs, mult, EOS,
                          n_rows=n_rows, hash_only=True)
    stride = addr.row_stride
    out = {}

    def timed(name, fn, nbytes, note):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(K):
            fn()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / K
        gbs = nbytes / (ms * 1e-3) / 1e9
        out[name] = {"ms": ms, "bytes": int(nbytes), "gbs": gbs, "frac": gbs / peak, "bytes_are": note}

    # engram_hash: 16 M positions of a Zipf stream, 16 heads each
    T = 1 << 24 if n_rows == FULL_ROWS else 1 << 22
    toks = zipf_tokens(torch, T, g, cdf)
    ids = torch.empty(T * 16, dtype=torch.int32, device=device)
    timed("engram_hash (k_hash)", lambda: L.check(lib.engram_hash(C.byref(addr.ctable), toks.data_ptr(), None, 0, T,
                                                                  ids.data_ptr(), stream), "engram_hash"),
          T * (4 + 64), "4 B token in + 16 x 4 B ids out per position")
    del ids
    # row sets over the 320 M-row table: a 40 MB bitmap (it fits in L2, as in the descent's own use)
    words = int(lib.engram_rowset_words(n_rows))
    bm_a = torch.zeros(words, dtype=torch.int32, device=device)
    bm_b = torch.zeros(words, dtype=torch.int32, device=device)
    bm_c = torch.empty(words, dtype=torch.int32, device=device)
    n_mark = 1 << 20
    timed("engram_rowset_mark (k_mark_positions)",
          lambda: L.check(lib.engram_rowset_mark(C.byref(addr.ctable), toks.data_ptr(), T, None, None, n_mark,
                                                 bm_a.data_ptr(), stream), "engram_rowset_mark"),
          n_mark * (4 + 16 * 4), "4 B token in + one 4 B bitmap word per head, per position")
    some = torch.randint(0, n_rows, (1 << 22,), generator=g, device=device, dtype=torch.int32)
    timed("engram_rowset_mark_ids (k_mark_ids)",
          lambda: L.check(lib.engram_rowset_mark_ids(some.data_ptr(), some.numel(), n_rows, bm_b.data_ptr(),
                                                     stream), "engram_rowset_mark_ids"),
          some.numel() * 8, "4 B id in + one 4 B bitmap word per id")
    timed("engram_rowset_combine (k_combine, union)",
          lambda: L.check(lib.engram_rowset_combine(bm_a.data_ptr(), bm_b.data_ptr(), words, 0, bm_c.data_ptr(),
                                                    stream), "engram_rowset_combine"),
          3 * words * 4, "two bitmaps read, one written")
    wsb = int(lib.engram_rowset_workspace_bytes(words))
    ws = torch.empty(wsb, dtype=torch.uint8, device=device)
    cnt = torch.zeros(1, dtype=torch.int64, device=device)
    lib.engram_rowset_extract(bm_c.data_ptr(), words, None, 0, cnt.data_ptr(), ws.data_ptr(), wsb, stream)
    torch.cuda.synchronize()
    members = int(cnt.item())
    mem_ids = torch.empty(members, dtype=torch.int32, device=device)
    timed("engram_rowset_extract (k_tile_*)",
          lambda: L.check(lib.engram_rowset_extract(bm_c.data_ptr(), words, mem_ids.data_ptr(), members,
                                                    cnt.data_ptr(), ws.data_ptr(), wsb, stream),
                          "engram_rowset_extract"),
          words * 4 + members * 4, "bitmap read + member ids written")
    ix = torch.empty(some.numel(), dtype=torch.int32, device=device)
    timed("engram_rowset_index (k_index)",
          lambda: L.check(lib.engram_rowset_index(bm_c.data_ptr(), words, ws.data_ptr(), wsb, some.data_ptr(),
                                                  some.numel(), ix.data_ptr(), stream), "engram_rowset_index"),
          some.numel() * (4 + 4 + 4 + 4), "per id: id in, bitmap word, prefix word, index out")
    del bm_a, bm_b, bm_c, ws, mem_ids, ix
    # engram_overlay_accumulate: one .pleo file of 400 k rows x 160 into a 1 M-row union, distinct and repeated rows
    n_ov, dim_ov, n_union = 400_000, 160, 1_000_000
    acc = torch.zeros(n_union, dim_ov, device=device)
    data = torch.randn(n_ov, dim_ov, generator=g, device=device)
    base = torch.randn(n_ov, dim_ov, generator=g, device=device)
    tgt = torch.randperm(n_union, generator=g, device=device)[:n_ov].to(torch.int32)
    timed("engram_overlay_accumulate (k_overlay_accumulate, distinct rows)",
          lambda: L.check(lib.engram_overlay_accumulate(acc.data_ptr(), tgt.data_ptr(), None, data.data_ptr(),
                                                        base.data_ptr(), n_ov, dim_ov, stream),
                          "engram_overlay_accumulate"),
          n_ov * dim_ov * 4 * 4 + n_ov * 4, "data, base and the target row read, target written (fp32)")
    tgt_rep = torch.randint(0, n_ov // 4, (n_ov,), generator=g, device=device, dtype=torch.int32)
    order = torch.sort(tgt_rep.long(), stable=True).indices
    timed("engram_overlay_accumulate (k_overlay_accumulate_runs, 4 rows per target)",
          lambda: L.check(lib.engram_overlay_accumulate(acc.data_ptr(), tgt_rep.data_ptr(), order.data_ptr(),
                                                        data.data_ptr(), base.data_ptr(), n_ov, dim_ov, stream),
                          "engram_overlay_accumulate"),
          n_ov * dim_ov * 4 * 2 + (n_ov // 4) * dim_ov * 4 * 2 + n_ov * 12,
          "data and base read, each distinct target read and written once, index and order read")
    del acc, data, base, tgt, tgt_rep, order
    # the row-sharded exchange at W = 4 (emulated on this GPU): config 5's batch of 131,072 positions
    W, me = 4, 1
    n5 = 64 * 2048
    region = n5 * 16
    tok5 = toks[:n5].contiguous()
    req_ids = [torch.empty(W * region, dtype=torch.int32, device=device) for _ in range(W)]
    req_cnt = [torch.zeros(W, dtype=torch.int64, device=device) for _ in range(W)]
    id_ptrs = torch.tensor([x.data_ptr() for x in req_ids], dtype=torch.int64, device=device)
    cnt_ptrs = torch.tensor([x.data_ptr() for x in req_cnt], dtype=torch.int64, device=device)
    counts = torch.zeros(W, dtype=torch.int64, device=device)
    rix = torch.empty(region, dtype=torch.int32, device=device)
    no_ov = L.EngramOverlay(None, 0, None, None, 0)
    timed("engram_shard_route_push (k_route_push + k_route_finish)",
          lambda: L.check(lib.engram_shard_route_push(C.byref(addr.ctable), C.byref(no_ov), tok5.data_ptr(), None, 0,
                                                      n5, W, me, id_ptrs.data_ptr(), cnt_ptrs.data_ptr(), region,
                                                      counts.data_ptr(), rix.data_ptr(), stream),
                          "engram_shard_route_push"),
          n5 * 4 + region * 4 * 2 + int(region * (W - 1) / W) * 4,
          "tokens in, row_index written then rewritten, one 4 B id per remote pair")
    n_local = (n_rows + W - 1) // W
    # one buffer of a W=2 shard's rows (23 GB): a W=4 owner's shard below, every owner's shard of the W=2 stage;
    # its contents do not change the timing
    shard = torch.empty(((n_rows + 1) // 2) * stride, dtype=torch.uint8, device=device)
    owner = (me + 1) % W
    for r in range(W):  # every other requester's ids of this batch for `owner`
        if r != owner:
            L.check(lib.engram_shard_route_push(C.byref(addr.ctable), C.byref(no_ov), tok5.data_ptr(), None, 0, n5,
                                                W, r, id_ptrs.data_ptr(), cnt_ptrs.data_ptr(), region,
                                                counts.data_ptr(), rix.data_ptr(), stream), "engram_shard_route_push")
    torch.cuda.synchronize()
    served = int(req_cnt[owner].sum().item()) - int(req_cnt[owner][owner].item())
    send = torch.empty(W * region * stride, dtype=torch.uint8, device=device)
    timed("engram_shard_serve_pushed (k_serve_pushed)",
          lambda: L.check(lib.engram_shard_serve_pushed(shard.data_ptr(), stride, n_local, W, owner,
                                                        req_ids[owner].data_ptr(), req_cnt[owner].data_ptr(), region,
                                                        send.data_ptr(), stream), "engram_shard_serve_pushed"),
          served * (4 + 2 * stride), "per served row: its id, the row read from the shard and written")
    del send, req_ids, rix
    # the legacy pulled stage at W = 2 (both owners' shards the same buffer, local rows g / 2 < its rows): rows of
    # the other rank copied in
    W2 = 2
    n_stage = 1 << 14
    shard_ptrs = torch.tensor([shard.data_ptr()] * W2, dtype=torch.int64, device=device)
    sb = int(lib.engram_stage_bytes(C.byref(addr.ctable), n_stage))
    stage = torch.empty(sb, dtype=torch.uint8, device=device)
    hid = torch.empty(n_stage * 16, dtype=torch.int32, device=device)
    L.check(lib.engram_hash(C.byref(addr.ctable), toks.data_ptr(), None, 0, n_stage, hid.data_ptr(), stream), "hash")
    torch.cuda.synchronize()
    remote = int(((hid.long() % W2) != 0).sum().item())
    timed("engram_stage_sharded (k_stage_sharded, W=2)",
          lambda: L.check(lib.engram_stage_sharded(C.byref(addr.ctable), C.byref(no_ov), toks.data_ptr(), None, 0,
                                                   n_stage, shard_ptrs.data_ptr(), W2, 0, stage.data_ptr(), 0, stream),
                          "engram_stage_sharded"),
          n_stage * 4 + remote * 2 * stride, "tokens in, each remote row read and written")
    del shard, stage, hid
    # PLE block backward at the reference's width: 2048 positions, hc = 4, n_embd = 2560
    hc, n, Kc, dil, Tp = 4, 2560, 4, 3, 2048
    r_ = lambda *sh: torch.randn(*sh, generator=g, device=device) * 0.1  # noqa: E731
    kvs = hc * n + n
    kv, hidden, dout, dnormed = r_(Tp, kvs), r_(Tp, hc, n), r_(Tp, hc, n), r_(Tp, hc, n)
    nk, nq, nc, conv_w = 1 + r_(hc * n), 1 + r_(hc * n), 1 + r_(hc * n), r_(hc * n, Kc)
    gate, s_ = torch.rand(Tp, hc, generator=g, device=device), r_(Tp, hc)
    normed, hist = r_(Tp, hc, n), r_((Kc - 1) * dil, hc, n)
    dkv, dhidden = torch.empty(Tp, kvs, device=device), torch.empty(Tp, hc, n, device=device)
    dconv, dnorm_out = torch.empty(Tp, hc, n, device=device), torch.empty(Tp, hc, n, device=device)
    Cb = Tp * hc * n * 4
    timed("engram_ple_gate_backward (k_ple_gate_bwd)",
          lambda: L.check(lib.engram_ple_gate_backward(
              kv.data_ptr(), kvs, kv[:, hc * n:].data_ptr(), kvs, hidden.data_ptr(), nk.data_ptr(), nq.data_ptr(),
              nc.data_ptr(), gate.data_ptr(), s_.data_ptr(), dout.data_ptr(), dnormed.data_ptr(), Tp, hc, n, 1e-6, 0, 0,
              dkv.data_ptr(), kvs, dkv[:, hc * n:].data_ptr(), kvs, dhidden.data_ptr(), stream),
              "engram_ple_gate_backward"),
          4 * Cb + Tp * n * 4 + 2 * Cb + Tp * n * 4,
          "key, hidden, dout, dnormed and value read; dkey, dhidden and dvalue written")
    timed("engram_ple_conv_backward (k_ple_dconv + k_ple_dx)",
          lambda: L.check(lib.engram_ple_conv_backward(
              normed.data_ptr(), hist.data_ptr(), hist.shape[0], conv_w.data_ptr(), Kc, dil, Tp, hc, n,
              dout.data_ptr(), None, 0, dconv.data_ptr(), dnorm_out.data_ptr(), None, stream),
              "engram_ple_conv_backward"),
          3 * Cb, "normed and dout read, dnormed written (the silu'-scaled gradient is a scratch pass)")
    line = {"metric": "per-kernel HBM GB/s of the kernels off the config-5 step",
            "unit": "GB/s", "peak_gbs": peak, "peak_source": peak_kind, "launches_timed": K, "kernels": out,
            "table_rows": n_rows,
            "config": {"workload": "micro: engram_hash over 16 M positions; row sets over the 320 M-row table; "
                                   "a 400 k x 160 .pleo accumulation; the pushed exchange at W=4 and the pulled "
                                   "stage at W=2 emulated on one GPU with config 5's batch; the PLE backward at "
                                   "2048 x hc 4 x 2560"}}
    print(json.dumps(line), flush=True)


def shard_text(cfg):
    if not cfg.get("shard"):
        return ""
    if cfg.get("stage") == "exchange":
        return ("+row-sharded table (id mod N; the rows of other ranks routed three batches ahead with their ids "
                "stored into the owners' memory, gathered by the owners and copied with the copy engines over "
                "NVLink; local rows read in place)")
    if cfg.get("shard_exchange", "peer") != "peer":
        return "+row-sharded table (id mod N, NCCL all-to-all of ids and rows)"
    if cfg.get("stage", "push") == "push":
        return ("+row-sharded table (id mod N; during the previous step each owner stores the rows it holds into "
                "the other ranks' stage buffers over NVLink, on a side stream; the forward reads local HBM)")
    if cfg.get("stage", "push") == "pull":
        return ("+row-sharded table (id mod N; the rows of other ranks are loaded from their owners over NVLink on a "
                "side stream during the previous step, the forward reads local HBM)")
    return "+row-sharded table (id mod N; rows read from their owners over NVLink inside the forward)"


def config_json(cfg, args):
    return {"workload": f"{args.config}: {cfg['seqs']}x{cfg['seq_len']} tokens/GPU, Zipf(1.1) over {VOCAB}, "
                        f"{cfg['rows']}-row x {cfg['dim']} {cfg['fmt']} table, R={cfg['R']} overlay rows, "
                        f"{cfg['mode']} emit, {'fwd+bwd+Adam' if cfg['bwd'] else 'fwd only'}",
            "table_rows": cfg["rows"], "dim": cfg["dim"], "format": cfg["fmt"], "positions_per_gpu": cfg["seqs"] * cfg["seq_len"],
            "overlay_rows": cfg["R"], "emit": cfg["mode"],
            "parallelism": f"dp{args.gpus}" + shard_text(cfg),
            "optimizer_exchange": (None if args.gpus == 1 else
                                   ("one peer-memory kernel per rank (sum over ranks + Adam + stores to every rank)"
                                    if cfg.get("exchange", "peer") == "peer" else "NCCL reduce-scatter + all-gather")),
            "l2": "inputs larger than L2 (residual and upstream gradient 537 MB each, table 46 GB)"}


START = time.perf_counter()


def main():
    args = parse()
    if args.config in ("scan", "ple", "micro"):
        import torch
        run = {"scan": run_scan, "ple": run_ple, "micro": run_micro}[args.config]
        run(args, torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0"))))
        return
    cfg = dict(CONFIGS[args.config])
    if args.table_rows:
        cfg["rows"] = args.table_rows
    if args.seqs:
        cfg["seqs"] = args.seqs
    world_env = int(os.environ.get("WORLD_SIZE", "1"))
    # config 5 at N > 1: the north star's layout (the table row-sharded, id mod N) is the headline by default
    cfg["shard"] = bool(args.shard) or (args.config == "cfg5" and world_env > 1 and args.layout == "sharded")
    cfg["exchange"] = args.exchange
    cfg["shard_exchange"] = args.shard_exchange
    cfg["stage"] = args.stage
    cfg["stage_blocks"] = args.stage_blocks
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.gpus > 1 and world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} needs torchrun with {args.gpus} ranks (WORLD_SIZE={world})")
    if args.impl == "reference":
        run_reference(args, cfg, rank)
        return
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
    wl = Workload(cfg, rank, world, args.seed, device)
    lib = wl.L.load()
    ddist = dist if world > 1 else None
    nbytes = wl.algorithmic_bytes()
    step_bytes = nbytes["fwd"] + nbytes["bwd"] + nbytes["adam"]
    parity = None
    if world == 1 and not args.no_check:
        parity = parity_check(wl)

    K = args.steps
    with ClockSampler(local) as clk:
        ms, fwd_ms, bwd_ms, launches = time_steps(wl, K, args.warmup, ddist)
    value = 16 * wl.n_out * world / (ms * 1e-3)
    n_out, pairsum = wl.n_out, wl.mode == wl.L.MODE_PAIRSUM_ADD_BF16

    e2e = None
    if not args.no_e2e and not wl.decode:
        e2e = run_e2e(wl, args, device, ddist, world)
    latency = None
    if world == 1 and args.config == "cfg5" and not args.no_latency:
        latency = run_latency(wl, args, device)

    layout = None
    if world > 1 and args.config == "cfg5":
        layout = {"headline": "row_sharded" if cfg["shard"] else "replicated"}
        if cfg["shard"]:
            layout["row_sharded"] = sharded_stats(wl, ms, fwd_ms, bwd_ms, ddist, world, device)
    if world > 1 and args.config == "cfg5" and not args.no_sharded_line:
        # the other layout, measured in the same run on the same batches; the two forwards are compared bit
        # for bit on this rank's batch (the overlay rows of the replicated run, the same residual)
        torch.cuda.synchronize()
        cfg2 = dict(cfg, shard=not cfg["shard"], stage="exchange")
        wl2 = Workload(cfg2, rank, world, args.seed, device)
        sh, rep = (wl, wl2) if cfg["shard"] else (wl2, wl)
        layout["sharded_vs_resident_forward"] = compare_layouts(sh, rep, ddist, device)
        if not cfg["shard"]:
            del wl
        ms2, fwd2, bwd2, _ = time_steps(wl2, K, args.warmup, ddist)
        side = {"value": 16 * wl2.n_out * world / (ms2 * 1e-3), "unit": "rows/s", "ms_per_step": ms2,
                "phase_ms": {"forward": fwd2, "backward": bwd2, "optimizer_and_exchange": ms2 - fwd2 - bwd2},
                "parallelism": f"dp{world}" + shard_text(cfg2)}
        if cfg2["shard"]:
            side.update(sharded_stats(wl2, ms2, fwd2, bwd2, ddist, world, device))
            layout["row_sharded"] = side
        else:
            layout["replicated"] = side

    if rank == 0:
        peak, peak_kind = measured_peak_gbs()
        fwd_gbs = nbytes["fwd"] / (fwd_ms * 1e-3) / 1e9
        traffic, tfile = profiled_traffic("k_forward_pairsum" if pairsum else "k_forward_concat")
        line = {
            "metric": METRIC, "value": value, "unit": "rows/s", "n_gpus": world, "steps": K, "warmup": args.warmup,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded Zipf tokens, random IQ4_XS table)",
            "config": config_json(cfg, args),
            "gbps": step_bytes * world / (ms * 1e-3) / 1e9,
            "algorithmic_bytes_per_step_per_gpu": step_bytes,
            "bytes_breakdown": nbytes,
            "hit_fraction": nbytes["hits"] / (16 * n_out),
            "phase_ms": {"forward": fwd_ms, "backward": bwd_ms, "optimizer_and_exchange": ms - fwd_ms - bwd_ms},
            "us_per_step": ms * 1e3,
            "roofline": {"kernel": "engram_forward (k_forward_pairsum_fixed<IQ4_XS,256>)" if pairsum else "engram_forward (k_forward_concat)",
                         "bound": "hbm", "achieved": fwd_gbs, "peak": peak, "unit": "GB/s", "frac": fwd_gbs / peak,
                         "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else "fallback 6650 GB/s",
                         "traffic": traffic, "traffic_source": tfile,
                         "traffic_note": ("DRAM read + write bytes per launch from the committed ncu capture of the same "
                                          "kernel on the same 131,072 positions with a 2^24-row table (a launch moves "
                                          "what its positions and rows need, whatever the table size), not measured "
                                          "in this run") if traffic is not None else None,
                         "algorithmic_bytes_per_launch": nbytes["fwd"],
                         "avg_launch_ms": fwd_ms},
            "gpu_launches": int(launches),
            "clocks": clk.summary(),
            "e2e": e2e,
        }
        if parity is not None:
            line["parity"] = parity
        if latency is not None:
            line["latency"] = latency
        if layout is not None:
            line["layouts"] = layout
        if world == 1 and not args.no_cpu_baseline:
            try:
                b = cpu_oracle_step_time(cfg, args.seed)
                line["cpu_baseline"] = {
                    "value": 16 * b["T_full"] / b["t_step"], "unit": "rows/s", "cores": b["threads"], "kind": "port",
                    "sample": f"oracle (C restatement of the reference path, OpenMP {b['threads']} threads) on "
                              f"{b['T_s']} Zipf positions of a {b['n_rows']}-row slice of the table, fwd+bwd "
                              f"{b['t_fb']:.3f}s extrapolated x{b['T_full'] / b['T_s']:.0f} plus Adam over "
                              f"{b['R']} rows {b['t_adam']:.3f}s (medians of {b['repeats']} repeats, "
                              f"{b['cpu_seconds']:.1f}s of CPU work)"}
            except Exception as exc:  # report, never hide, a failed baseline
                line["cpu_baseline"] = {"value": None, "error": repr(exc)[:200]}
        print(json.dumps(line), flush=True)
    if ddist is not None:
        dist.barrier()
        dist.destroy_process_group()


def sharded_stats(wl, ms, fwd_ms, bwd_ms, ddist, world, device):
    """What the row-sharded table moves per step (max over ranks): the (position,
    head) pairs served by other ranks, the distinct rows among them (the rows
    the exchange carries) and their bytes over NVLink."""
    import torch
    rr = torch.tensor([wl.remote_rows, wl.remote_distinct], dtype=torch.int64, device=device)
    ddist.all_reduce(rr, op=ddist.ReduceOp.MAX)
    nv_bytes = int(rr[0]) * wl.shard.stride  # the exchange moves one row per remote (position, head) pair
    phases = None
    xs = getattr(wl.shard, "xstage", None)
    if xs is not None:  # more steps with the exchange's phases timed (after the timed region and 3 plain steps)
        import torch
        for _ in range(3):
            wl.step(ddist)
        xs.timing = {}
        for _ in range(9):
            wl.step(ddist)
        wl.join_stage()
        torch.cuda.synchronize()
        ph = xs.phase_ms()
        xs.timing = None
        keys = sorted(ph)
        t = torch.tensor([ph[k] for k in keys], dtype=torch.float64, device=device)
        ddist.all_reduce(t, op=ddist.ReduceOp.MAX)
        phases = {k: float(v) for k, v in zip(keys, t.tolist())}
        phases["note"] = ("ms per step, the median of 9 steps, max over ranks: route (ids pushed to their owners), serve (the owner's "
                          "local gather) and barrier (a 4-byte all-reduce) on the step's stream before the forward, "
                          "fetch (copy-engine transfers) on the side stream, wait = the forward's stream blocked on "
                          "its rows")
    return {"table_bytes_per_gpu": int(wl.shard.n_local * wl.shard.stride), "exchange_phase_ms": phases,
            "nvlink": {"remote_pairs_per_step": int(rr[0]), "distinct_remote_rows_per_step": int(rr[1]),
                       "dedup_factor": int(rr[0]) / max(int(rr[1]), 1), "bytes_per_step": nv_bytes,
                       "achieved_gbps": nv_bytes / (ms * 1e-3) / 1e9, "peer_copy_gbps": 770.0,
                       "frac_of_peer_copy": nv_bytes / (ms * 1e-3) / 1e9 / 770.0}}


def compare_layouts(sh, rep, ddist, device):
    """The row-sharded forward (a shard of the replicated run's table, this
    rank's rows, with the same exchange staging as the timed run) against the
    forward over the whole resident table, on this rank's batch, with the
    replicated run's overlay rows and the same residual: bf16 bits, slots and
    hit counts compared on the device (mismatches summed over ranks)."""
    import ctypes as C
    import torch
    from engraft_ngram_b200.shard import ShardedTable
    L = rep.L
    world, rank = rep.world, rep.rank
    shard = ShardedTable.from_full(rep.table, world, rank)
    shard.enable_exchange_staging(rep.T)
    res0 = rep.out.clone()
    a, b = res0.clone(), res0.clone()
    sa = torch.empty_like(rep.slots)
    sb = torch.empty_like(rep.slots)
    ha = torch.zeros(1, dtype=torch.int64, device=device)
    hb = torch.zeros(1, dtype=torch.int64, device=device)
    tok = rep.tokens.clone()
    shard.forward(tok, rep.seg_start, rep.omap, rep.rows_var, a, rep.mode, slots_out=sa, hit_count=ha)
    ov = rep.omap.descriptor(rep.rows_var)
    st = L.load().engram_forward(C.byref(rep.table.ctable), C.byref(ov), tok.data_ptr(), rep.seg_start.data_ptr(), 0,
                                 rep.T, rep.mode, b.data_ptr(), None, sb.data_ptr(), hb.data_ptr(), rep.stream)
    L.check(st, "engram_forward")
    mism = torch.stack([(a.view(torch.int16) != b.view(torch.int16)).sum(), (sa != sb).sum(), (ha != hb).sum()])
    checked = torch.tensor([a.numel(), sa.numel()], dtype=torch.int64, device=device)
    ddist.all_reduce(mism)
    ddist.all_reduce(checked)
    torch.cuda.synchronize()
    del res0, shard
    return {"residual_values": int(checked[0]), "slots": int(checked[1]), "mismatches": int(mism.sum()),
            "bit_exact": int(mism.sum()) == 0}


def time_steps(wl, K, warmup, ddist):
    """max(3, warmup) untimed steps, then K steps between CUDA events on the
    launching stream, bracketed by a barrier and a synchronize; the step time
    and the forward time are maxima over ranks.  Returns (ms per step, forward
    ms, backward ms, kernel launches in the timed region)."""
    import torch
    lib = wl.L.load()
    bwd = wl.cfg["bwd"] and wl.R
    for _ in range(max(3, warmup)):
        wl.step(ddist)
    torch.cuda.synchronize()
    f0 = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    f1 = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    b1 = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if ddist is not None:
        ddist.barrier()
    torch.cuda.synchronize()
    n_launch0 = lib.engram_launch_count()
    e0.record()
    for k in range(K):
        f0[k].record()
        wl.forward()
        f1[k].record()
        if bwd:
            wl.backward()
            b1[k].record()
            wl.optimizer(ddist)
    if wl.stage:  # the copy for the step after the last is timed too
        wl.join_stage()
    e1.record()
    torch.cuda.synchronize()
    launches = lib.engram_launch_count() - n_launch0
    if ddist is not None:
        ddist.barrier()
    ms = e0.elapsed_time(e1) / K
    fwd_ms = sum(a.elapsed_time(b) for a, b in zip(f0, f1)) / K
    bwd_ms = sum(a.elapsed_time(b) for a, b in zip(f1, b1)) / K if bwd else 0.0
    t = torch.tensor([ms, fwd_ms, bwd_ms], device=wl.dev, dtype=torch.float64)
    if ddist is not None:
        ddist.all_reduce(t, op=ddist.ReduceOp.MAX)
    return float(t[0]), float(t[1]), float(t[2]), int(launches)


def run_e2e(wl, args, device, ddist, world):
    """Same step through the public Python API with host inputs: tokens and
    segment starts copied from pinned host memory each step, the hit count
    copied back to pinned host memory each step.  The host reads a step's hit
    count while the next step runs (it waits on the step's event one step
    later, as a training loop that logs the previous step does), so the host's
    launch work overlaps the GPU's; the last count is read after the timed
    loop's final synchronize."""
    import torch
    eb = wl.eb
    K = max(1, min(args.steps, 200))
    tok_h = wl.tokens.cpu().pin_memory()
    ss_h = wl.seg_start.cpu().pin_memory()
    hit_h = [torch.zeros(1, dtype=torch.int64).pin_memory() for _ in range(2)]
    done = [None, None]
    counter = [0]
    if wl.peer is not None and args.e2e_exchange == "peer":  # autograd backward into the owners (PeerRows.attach)
        from engraft_ngram_b200.dist import PeerAdam
        wl.peer.rows_var.copy_(wl.p0)
        rows_var = wl.peer.rows_var.requires_grad_(True)
        wl.peer.attach(wl.omap)
        opt = PeerAdam(wl.peer, lr=wl.lr, reg_ref=wl.p0, reg_mu=wl.mu)
        api = "engraft_ngram_b200.engram_residual_add + autograd backward into PeerRows + PeerAdam.step"
    else:
        rows_var = wl.p0.clone().requires_grad_(True)
        opt = eb.OverlayAdam([rows_var], lr=wl.lr, reg_ref=wl.p0, reg_mu=wl.mu)
        api = ("engraft_ngram_b200.engram_residual_add + autograd backward + "
               + ("NCCL all-reduce of the row gradients + " if ddist is not None else "") + "OverlayAdam.step")
    hits = torch.zeros(1, dtype=torch.int64, device=device)
    pending = []  # the next steps' inputs, copied (and for sharded reads prefetched) ahead
    h2d = torch.cuda.Stream(device)  # the token copies, apart from the exchange's row copies

    def one():
        residual = wl.out.detach()
        if wl.stage:  # this step's inputs were copied and prefetched wl.depth steps ago
            while len(pending) < wl.depth:
                pending.append((tok_h.to(device, non_blocking=True), ss_h.to(device, non_blocking=True)))
            tok, ss = pending.pop(0)
            xs = getattr(wl.table, "xstage", None)
            if xs is not None:  # copied on a stream of their own: the exchange waits for the copy, not for the step
                with torch.cuda.stream(h2d):
                    nxt = (tok_h.to(device, non_blocking=True), ss_h.to(device, non_blocking=True))
                    ready = torch.cuda.Event()
                    ready.record(h2d)
                for x in nxt:
                    x.record_stream(torch.cuda.current_stream(device))
                wl.table.prefetch(nxt[0], nxt[1], omap=wl.omap, ready=ready)
            else:
                nxt = (tok_h.to(device, non_blocking=True), ss_h.to(device, non_blocking=True))
                wl.table.prefetch(nxt[0], nxt[1], max_blocks=wl.stage_blocks, omap=wl.omap)
            pending.append(nxt)
        else:  # copied one step ahead on a stream of their own: the copy overlaps the step before
            cur = torch.cuda.current_stream(device)
            while len(pending) < 2:
                with torch.cuda.stream(h2d):
                    nxt = (tok_h.to(device, non_blocking=True), ss_h.to(device, non_blocking=True))
                    ready = torch.cuda.Event()
                    ready.record(h2d)
                for x in nxt:
                    x.record_stream(cur)
                pending.append((nxt[0], nxt[1], ready))
            tok, ss, ready = pending.pop(0)
            cur.wait_event(ready)
        hits.zero_()
        opt.zero_grad()
        if wl.mode == wl.L.MODE_PAIRSUM_ADD_BF16:
            out = eb.engram_residual_add(residual, wl.table, tok, rows_var, wl.omap, ss, 0, hits)
        else:
            out = eb.engram_embed(wl.table, tok, rows_var, wl.omap, ss, 0, wl.T, hits)
        if wl.cfg["bwd"] and wl.R:
            out.backward(wl.dout.reshape(out.shape))
            if ddist is not None and rows_var.grad is not None:
                ddist.all_reduce(rows_var.grad)
            opt.step()
        b = counter[0] % 2
        counter[0] += 1
        hit_h[b].copy_(hits, non_blocking=True)
        done[b] = torch.cuda.Event()
        done[b].record(torch.cuda.current_stream(device))
        prev = done[b ^ 1]
        if prev is None:
            return None
        prev.synchronize()  # the previous step's result, read while this step runs
        return int(hit_h[b ^ 1].item())

    for _ in range(3):
        one()
    if ddist is not None:
        ddist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(K):
        one()
    if wl.stage:
        wl.join_stage()
    e1.record()
    torch.cuda.synchronize()
    last = int(hit_h[(counter[0] - 1) % 2].item())
    if last <= 0 and wl.R:
        raise RuntimeError("e2e: the last step reported no overlay hits")
    ms = e0.elapsed_time(e1) / K
    t = torch.tensor([ms], device=device, dtype=torch.float64)
    if ddist is not None:
        ddist.all_reduce(t, op=ddist.ReduceOp.MAX)
    ms = float(t[0])
    return {"value": 16 * wl.T * world / (ms * 1e-3), "unit": "rows/s", "ms_per_step": ms, "steps": K,
            "h2d_bytes_per_step": 8 * wl.T, "d2h_bytes_per_step": 8, "api": api}


if __name__ == "__main__":
    main()
