"""Multi-GPU plumbing for the overlay update: one process per GPU, data-parallel
over the token batch, the resident table replicated on every rank.

The path's only exchange step is the overlay gradient.  Every rank computes
row gradients for all R overlay rows from its own batch; the rows are then
sharded by contiguous blocks (rank r owns rows [r*R/W, (r+1)*R/W)):
  1. reduce-scatter of grad_rows [R, D] -> each owner's summed shard;
  2. the owner runs the fused Adam step (with the regulariser) on its shard;
  3. all-gather of the updated shards -> every rank's rows_var for the next
     forward.
Collectives go through torch.distributed (NCCL between GPUs, gloo on CPU for
tests).  The reference has no multi-GPU code; W=1 is bit-identical to the
single-process step, W>1 sums the per-rank gradients in rank order.
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist


def symmetric_memory():
    """torch's symmetric-memory module, with NVLink multicast turned off.

    The kernels of this package read and write peer buffers with plain loads,
    cp.async and plain stores only; none issues a multicast operation.  With
    TORCH_SYMM_MEM_DISABLE_MULTICAST=1 torch maps each buffer into the other
    ranks' processes without binding it to an NVLink multicast object, so a
    rank that ends while it holds such a buffer leaves no multicast object
    behind for the other GPUs.  The switch is set before every allocation
    this package makes, so it holds whichever allocation comes first."""
    os.environ["TORCH_SYMM_MEM_DISABLE_MULTICAST"] = "1"
    import torch.distributed._symmetric_memory as symm
    return symm


def shard_bounds(R: int, world: int, rank: int) -> tuple[int, int]:
    """Rows [lo, hi) of the overlay owned by `rank` (contiguous, near-equal)."""
    if world < 1 or not (0 <= rank < world):
        raise ValueError(f"bad rank {rank} of {world}")
    base, extra = divmod(R, world)
    lo = rank * base + min(rank, extra)
    hi = lo + base + (1 if rank < extra else 0)
    return lo, hi


def _equal_shards(R: int, world: int) -> bool:
    return R % world == 0


def reduce_scatter_rows(grad_rows: torch.Tensor, group=None) -> torch.Tensor:
    """Sum of grad_rows over ranks, restricted to this rank's shard."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    R = grad_rows.shape[0]
    lo, hi = shard_bounds(R, world, rank)
    if world == 1:
        return grad_rows[lo:hi]
    if _equal_shards(R, world) and dist.get_backend(group) == "nccl":
        out = torch.empty_like(grad_rows[lo:hi])
        dist.reduce_scatter_tensor(out, grad_rows.contiguous(), group=group)
        return out
    full = grad_rows.clone()
    dist.all_reduce(full, group=group)  # backends without reduce-scatter (gloo), or ragged shards
    return full[lo:hi]


def all_gather_rows(rows_var: torch.Tensor, shard: torch.Tensor, group=None) -> None:
    """rows_var[all] <- the owners' shards (in place)."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    R = rows_var.shape[0]
    if world == 1:
        lo, hi = shard_bounds(R, 1, 0)
        if shard.data_ptr() != rows_var[lo:hi].data_ptr():
            rows_var[lo:hi].copy_(shard)
        return
    if _equal_shards(R, world) and dist.get_backend(group) == "nccl":
        lo, hi = shard_bounds(R, world, rank)
        if shard.data_ptr() != rows_var[lo:hi].data_ptr():
            rows_var[lo:hi].copy_(shard)
        dist.all_gather_into_tensor(rows_var, rows_var[lo:hi], group=group)
        return
    # ragged shards or a backend without all_gather_into_tensor: pad every shard to the largest
    spans = [shard_bounds(R, world, r) for r in range(world)]
    width = max(hi - lo for lo, hi in spans)
    padded = torch.zeros((width,) + tuple(rows_var.shape[1:]), dtype=rows_var.dtype, device=rows_var.device)
    padded[: shard.shape[0]].copy_(shard)
    parts = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(parts, padded, group=group)
    for (lo, hi), part in zip(spans, parts):
        rows_var[lo:hi].copy_(part[: hi - lo])


def backward_to_owners(slots: torch.Tensor, grad: torch.Tensor, n_heads: int, hpn: int, dim: int, R: int, mode: int,
                       owner_ptrs: torch.Tensor, world: int, rank: int, workspace: torch.Tensor | None = None) -> None:
    """engram_backward_to_owners: this rank's row gradients, each row stored
    into its owner's receive buffer (block `rank`)."""
    from . import _lib as L
    lib = L.load()
    n = slots.shape[0]
    ws_bytes = int(lib.engram_backward_workspace_bytes(n, n_heads, R))
    L.check(min(ws_bytes, 0), "engram_backward_workspace_bytes")
    if workspace is None or workspace.numel() < ws_bytes:
        workspace = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=slots.device)
    st = lib.engram_backward_to_owners(slots.data_ptr(), n, n_heads, hpn, mode, grad.data_ptr(), dim, R,
                                       owner_ptrs.data_ptr(), world, rank, workspace.data_ptr(), workspace.numel(),
                                       L.stream_of(slots.device))
    L.check(st, "engram_backward_to_owners")


def adam_owner_step(recv: torch.Tensor, rows_ptrs: torch.Tensor, world: int, rank: int, R: int, dim: int,
                    m: torch.Tensor, v: torch.Tensor, p0: torch.Tensor | None, step: int, lr: float,
                    beta1: float = 0.9, beta2: float = 0.999, eps: float = 1e-8, reg_scale: float = 0.0) -> None:
    """engram_adam_owner_step: sum of the receive buffer's blocks in rank order,
    Adam on this rank's rows (m, v, p0: the owned rows), stores into every
    rank's rows_var."""
    from . import _lib as L
    st = L.load().engram_adam_owner_step(recv.data_ptr(), rows_ptrs.data_ptr(), world, rank, R, dim, m.data_ptr(),
                                         v.data_ptr(), L.ptr(p0), int(step), float(lr), float(beta1), float(beta2),
                                         float(eps), float(reg_scale), L.stream_of(m.device))
    L.check(st, "engram_adam_owner_step")


class PeerRows:
    """The data-parallel overlay update over peer memory.  rows_var [R, dim] and
    a receive buffer [world, ceil(R/world), dim] live in torch symmetric memory,
    so every rank's copies are mapped into every process over NVLink.  Per step:
      backward(): the row gradients go straight to their owners' receive
        buffers (the reduce-scatter's transfer, inside the reduction);
      step(): barrier; each owner sums its blocks in rank order, runs Adam and
        stores the new rows into every rank's rows_var (the all-gather's
        transfer, inside the update); barrier.
    The barriers are tiny NCCL all-reduces on the stream; no kernel waits on
    another GPU."""

    def __init__(self, R: int, dim: int, device, group=None):
        symm = symmetric_memory()
        if dim % 4:
            raise ValueError("PeerRows needs dim % 4 == 0 (16-byte row pieces)")
        self.group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        self.R, self.dim = int(R), int(dim)
        chk = torch.tensor([self.R, -self.R, self.dim, -self.dim], dtype=torch.int64, device=device)
        dist.all_reduce(chk, op=dist.ReduceOp.MAX, group=self.group)
        if int(chk[0]) != -int(chk[1]) or int(chk[2]) != -int(chk[3]):
            raise ValueError(f"PeerRows: every rank needs the same R and dim (this rank: R={self.R}, dim={self.dim})")
        size_max = -(-self.R // self.world)
        self.recv = symm.empty(max(self.world * size_max, 1), self.dim, dtype=torch.float32, device=device)
        self.rows_var = symm.empty(max(self.R, 1), self.dim, dtype=torch.float32, device=device)
        self._hv = symm.rendezvous(self.recv, self.group)
        self._hr = symm.rendezvous(self.rows_var, self.group)
        self.recv_ptrs = torch.tensor(list(self._hv.buffer_ptrs), dtype=torch.int64, device=device)
        self.rows_ptrs = torch.tensor(list(self._hr.buffer_ptrs), dtype=torch.int64, device=device)
        self._flag = torch.zeros(1, dtype=torch.int32, device=device)
        self._ws = None

    def barrier(self) -> None:
        dist.all_reduce(self._flag, group=self.group)

    def backward(self, slots: torch.Tensor, grad: torch.Tensor, n_heads: int, hpn: int, mode: int) -> None:
        from . import _lib as L
        n = slots.shape[0]
        ws_bytes = int(L.load().engram_backward_workspace_bytes(n, n_heads, self.R))
        if self._ws is None or self._ws.numel() < ws_bytes:
            self._ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=slots.device)
        backward_to_owners(slots, grad, n_heads, hpn, self.dim, self.R, mode, self.recv_ptrs, self.world, self.rank,
                           self._ws)

    def step(self, m: torch.Tensor, v: torch.Tensor, p0: torch.Tensor | None, step: int, lr: float,
             beta1: float = 0.9, beta2: float = 0.999, eps: float = 1e-8, reg_scale: float = 0.0) -> None:
        self.barrier()
        adam_owner_step(self.recv, self.rows_ptrs, self.world, self.rank, self.R, self.dim, m, v, p0, step, lr,
                        beta1, beta2, eps, reg_scale)
        self.barrier()

    def attach(self, omap) -> None:
        """Route the autograd backward of engram_embed / engram_residual_add
        through this exchange: when they are given self.rows_var and `omap`,
        the row gradients go straight into the owners' receive buffers (as
        backward()) and rows_var.grad is left unset; PeerAdam steps the rows."""
        if omap.R != self.R:
            raise ValueError(f"overlay map has {omap.R} rows, the exchange {self.R}")
        omap.peer = self


class PeerAdam:
    """The data-parallel counterpart of OverlayAdam over a PeerRows exchange:
    same hyper-parameters and regulariser (reg_ref = the starting rows of all
    R rows, reg_mu), Adam moments kept for this rank's rows only; step() is
    PeerRows.step (barrier, owner sum + Adam + stores into every rank,
    barrier), a collective.  The row gradients come from the backward of a
    forward over peer.rows_var with the map attached (PeerRows.attach)."""

    def __init__(self, peer: PeerRows, lr: float = 1e-3, betas=(0.9, 0.999), eps: float = 1e-8,
                 reg_ref: torch.Tensor | None = None, reg_mu: float = 0.0):
        from .optim import reg_scale
        if lr < 0 or eps < 0 or not (0 <= betas[0] < 1 and 0 <= betas[1] < 1):
            raise ValueError(f"invalid Adam hyper-parameters lr={lr} betas={betas} eps={eps}")
        self.peer, self.lr, self.betas, self.eps = peer, float(lr), tuple(betas), float(eps)
        lo, hi = shard_bounds(peer.R, peer.world, peer.rank)
        dev = peer.rows_var.device
        self.m = torch.zeros(max(hi - lo, 1), peer.dim, device=dev)
        self.v = torch.zeros(max(hi - lo, 1), peer.dim, device=dev)
        self.reg_scale = reg_scale(reg_mu, reg_ref) if reg_ref is not None and reg_mu != 0.0 else 0.0
        self.p0 = reg_ref[lo:hi].detach().contiguous() if self.reg_scale != 0.0 else None
        self.t = 0

    def zero_grad(self, set_to_none: bool = True) -> None:
        """Nothing to clear: every backward rewrites all of this rank's blocks."""

    def step(self) -> None:
        self.t += 1
        self.peer.step(self.m, self.v, self.p0, self.t, self.lr, self.betas[0], self.betas[1], self.eps,
                       self.reg_scale)
