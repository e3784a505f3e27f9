"""Fused optimizer step over the overlay rows (K4).

`OverlayAdam` is a torch.optim.Optimizer with the constructor and update rule
of torch.optim.Adam as the descent uses it (engraft/descend_corpus.py:789-790:
default betas and eps, no weight decay), with the step done by one CUDA kernel
per parameter (engram_adam_step).  Given `reg_ref` (the starting rows p0) and
`reg_mu`, the kernel also adds the gradient of the descent's regulariser
mu * sum((p-p0)^2) / max(sum(p0^2), 1e-12) (engraft/descend_corpus.py:935-937),
so a caller can drop the separate `reg.backward()`.
"""
from __future__ import annotations

import torch

from . import _lib as L


def reg_scale(mu: float, p0: torch.Tensor) -> float:
    """float32(mu) / max(sum(p0^2), 1e-12): the factor autograd of the
    regulariser applies to 2*(p - p0)."""
    S = p0.detach().float().pow(2).sum().clamp_min(1e-12)
    return float((torch.tensor(float(mu), dtype=torch.float32, device=S.device) / S).item())


class OverlayAdam(torch.optim.Optimizer):
    def __init__(self, params, lr: float = 1e-3, betas=(0.9, 0.999), eps: float = 1e-8,
                 reg_ref: torch.Tensor | None = None, reg_mu: float = 0.0):
        if lr < 0 or eps < 0 or not (0 <= betas[0] < 1 and 0 <= betas[1] < 1):
            raise ValueError(f"invalid Adam hyper-parameters lr={lr} betas={betas} eps={eps}")
        super().__init__(params, dict(lr=lr, betas=tuple(betas), eps=eps))
        self.reg_ref = reg_ref
        self.reg_mu = float(reg_mu)
        self._reg_scale = reg_scale(reg_mu, reg_ref) if reg_ref is not None and reg_mu != 0.0 else 0.0

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        lib = L.load()
        for group in self.param_groups:
            b1, b2 = group["betas"]
            for p in group["params"]:
                if p.grad is None and self.reg_ref is None:
                    continue
                if not p.is_cuda or p.dtype != torch.float32 or not p.is_contiguous():
                    raise RuntimeError("OverlayAdam needs contiguous float32 CUDA parameters")
                g = p.grad if p.grad is not None else torch.zeros_like(p)
                g = g.contiguous()
                st = self.state[p]
                if not st:
                    st["step"] = 0
                    st["exp_avg"] = torch.zeros_like(p, memory_format=torch.contiguous_format)
                    st["exp_avg_sq"] = torch.zeros_like(p, memory_format=torch.contiguous_format)
                st["step"] += 1
                p0 = None
                rs = 0.0
                if self.reg_ref is not None and self._reg_scale != 0.0:
                    p0 = self.reg_ref.detach().contiguous()
                    if p0.shape != p.shape:
                        raise ValueError("reg_ref must have the parameter's shape")
                    rs = self._reg_scale
                s = lib.engram_adam_step(p.data_ptr(), g.data_ptr(), st["exp_avg"].data_ptr(),
                                         st["exp_avg_sq"].data_ptr(), L.ptr(p0), p.numel(), st["step"],
                                         float(group["lr"]), float(b1), float(b2), float(group["eps"]), float(rs),
                                         L.stream_of(p.device))
                L.check(s, "engram_adam_step")
        return loss
