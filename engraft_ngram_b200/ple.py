"""The PLE block that consumes the gathered rows, on the GPU: the drop-in for
`engraft.replica.layers.ple_forward` (engraft/replica/layers.py:565-626), same
arguments and results.

The key and value projections are one GEMM against [w_key; w_value].
PROJECTION selects its arithmetic and engine:
  "tcgen05": this library's own tensor-core GEMM (engram_gemm_3xtf32: tcgen05
    MMAs fed by TMA, the accumulator in tensor memory, the three 3xTF32
    products issued from one load of each operand slice), fp32 accumulation;
  "3xtf32" (default): each fp32 operand split into a TF32 head and the fp32
    remainder, x = hi + lo, and A B = hi_A hi_B + hi_A lo_B + lo_A hi_B on the
    tensor cores (the split-precision method of NVIDIA's CUTLASS "3xTF32"),
    with fp32 accumulation: fp32-level accuracy at tensor-core speed;
  "fp32": plain fp32 SGEMM (TF32 off), the reference's own arithmetic.
Everything after the projections is two kernels of this library:
engram_ple_gate (grouped RMS norms, the sign-sqrt sigmoid gate and the norm of
the gated value, one block per position) and engram_ple_conv (the causal
dilated depthwise conv over [history; positions], silu and the block's residual
sum).  Results agree with the reference to fp32 rounding (different reduction
orders).

Backward: calls that need gradients of emb, hidden or hist (what the descent's
loss.backward() differentiates, engraft/replica/seq.py:1457-1462) run through
an autograd function whose backward is engram_ple_conv_backward (silu' and the
transposed conv), engram_ple_gate_backward (the norms, the gate and the gated
product in closed form) and one GEMM back through both projections, d_emb =
[d_key, d_value] @ [w_key; w_value], in the forward's arithmetic.  Gradients of
the block's weights (frozen in the descent) are not built: such a call raises,
and `install_ple` routes it to the reference's own function.
"""
from __future__ import annotations

import contextlib
import ctypes as C

import torch

from . import _lib as L

_GRAD_FIELDS = ("w_key", "w_value", "norm_key", "norm_query", "norm_conv", "conv1d")
PROJECTION = "3xtf32"  # or "fp32", "tcgen05"


@contextlib.contextmanager
def _matmul_tf32(on: bool):
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = on
    try:
        yield
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def split_tf32(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """x = hi + lo exactly: hi keeps the 10 explicit mantissa bits TF32 holds
    (the low 13 bits cleared), lo = x - hi is the fp32 remainder."""
    hi = (x.contiguous().view(torch.int32) & -8192).view(torch.float32)
    return hi, x - hi


def _weights_kv(w, mode: str):
    """[w_key; w_value] and, for 3xtf32, its split, cached on `w` until a weight changes."""
    key = (mode, w.w_key.data_ptr(), w.w_key._version, w.w_value.data_ptr(), w.w_value._version)
    cached = getattr(w, "_engram_b200_kv", None)
    if cached is not None and cached[0] == key:
        return cached[1]
    kv = torch.cat([w.w_key, w.w_value], dim=0).contiguous()
    parts = split_tf32(kv) if mode == "3xtf32" else (kv,)
    try:
        setattr(w, "_engram_b200_kv", (key, parts))
    except AttributeError:  # a weights object without attributes of its own: no cache
        pass
    return parts


def gemm_tf32(terms, out: torch.Tensor, err: torch.Tensor | None = None) -> torch.Tensor:
    """out [M, N] = sum of A @ B.T over the (A [M, K], B [N, K]) pairs in terms,
    on the tensor cores (engram_gemm_tf32); fp32 contiguous CUDA tensors."""
    M, K = terms[0][0].shape
    N = terms[0][1].shape[0]
    a = (C.c_void_p * len(terms))(*[x.data_ptr() for x, _ in terms])
    b = (C.c_void_p * len(terms))(*[y.data_ptr() for _, y in terms])
    st = L.load().engram_gemm_tf32(len(terms), a, b, M, N, K, K, K, out.data_ptr(), out.stride(0), L.ptr(err),
                                   L.stream_of(out.device))
    L.check(st, "engram_gemm_tf32")
    return out


def gemm_3xtf32(a_hi, a_lo, b_hi, b_lo, out: torch.Tensor, err: torch.Tensor | None = None) -> torch.Tensor:
    """out [M, N] = (a_hi + a_lo) @ (b_hi + b_lo).T in 3xTF32 (the lo @ lo term
    dropped), every K slice of the four operands loaded once (engram_gemm_3xtf32)."""
    M, K = a_hi.shape
    N = b_hi.shape[0]
    st = L.load().engram_gemm_3xtf32(a_hi.data_ptr(), a_lo.data_ptr(), b_hi.data_ptr(), b_lo.data_ptr(), M, N, K,
                                     a_hi.stride(0), b_hi.stride(0), out.data_ptr(), out.stride(0), L.ptr(err),
                                     L.stream_of(out.device))
    L.check(st, "engram_gemm_3xtf32")
    return out


def _weights_t(w):
    """[w_key; w_value].T ([n, hc*n + n], K-major for the backward's GEMM) split
    into TF32 head and remainder, cached on `w` until a weight changes."""
    key = (w.w_key.data_ptr(), w.w_key._version, w.w_value.data_ptr(), w.w_value._version)
    cached = getattr(w, "_engram_b200_kvt", None)
    if cached is not None and cached[0] == key:
        return cached[1]
    parts = split_tf32(torch.cat([w.w_key, w.w_value], dim=0).t().contiguous())
    try:
        setattr(w, "_engram_b200_kvt", (key, parts))
    except AttributeError:
        pass
    return parts


def project(emb: torch.Tensor, w, out: torch.Tensor, mode: str | None = None) -> torch.Tensor:
    """out [T, hc*n + n] = emb @ [w_key; w_value].T (key columns, then value)."""
    mode = mode or PROJECTION
    if mode == "tcgen05":
        b_hi, b_lo = _weights_kv(w, "3xtf32")
        a_hi, a_lo = split_tf32(emb)
        return gemm_3xtf32(a_hi, a_lo, b_hi, b_lo, out)
    if mode == "fp32":
        (kv,) = _weights_kv(w, "fp32")
        with _matmul_tf32(False):
            torch.matmul(emb, kv.t(), out=out)
        return out
    if mode != "3xtf32":
        raise ValueError(f"projection mode {mode!r}")
    b_hi, b_lo = _weights_kv(w, "3xtf32")
    a_hi, a_lo = split_tf32(emb)
    with _matmul_tf32(True):
        torch.matmul(a_lo, b_hi.t(), out=out)  # the small terms first
        out.addmm_(a_hi, b_lo.t())
        out.addmm_(a_hi, b_hi.t())
    return out


def needs_grad(emb: torch.Tensor, hidden: torch.Tensor, w, hist: torch.Tensor) -> bool:
    if not torch.is_grad_enabled():
        return False
    ts = [emb, hidden, hist] + [getattr(w, f) for f in _GRAD_FIELDS]
    return any(isinstance(t, torch.Tensor) and t.requires_grad for t in ts)


def weights_need_grad(w) -> bool:
    """The block's weights need gradients (not built here)."""
    return torch.is_grad_enabled() and any(isinstance(getattr(w, f), torch.Tensor) and getattr(w, f).requires_grad
                                           for f in _GRAD_FIELDS)


def project_back(dkv: torch.Tensor, w, out: torch.Tensor, mode: str | None = None) -> torch.Tensor:
    """out [T, n] = dkv [T, hc*n + n] @ [w_key; w_value]: the gradient of emb
    through both projections, in the same arithmetic as project()."""
    mode = mode or PROJECTION
    if mode == "tcgen05":
        b_hi, b_lo = _weights_t(w)
        a_hi, a_lo = split_tf32(dkv)
        return gemm_3xtf32(a_hi, a_lo, b_hi, b_lo, out)
    if mode == "fp32":
        (kv,) = _weights_kv(w, "fp32")
        with _matmul_tf32(False):
            torch.matmul(dkv, kv, out=out)
        return out
    if mode != "3xtf32":
        raise ValueError(f"projection mode {mode!r}")
    b_hi, b_lo = _weights_kv(w, "3xtf32")
    a_hi, a_lo = split_tf32(dkv)
    with _matmul_tf32(True):
        torch.matmul(a_lo, b_hi, out=out)
        out.addmm_(a_hi, b_lo)
        out.addmm_(a_hi, b_hi)
    return out


def _block_forward(emb, hidden, w, hist, nk, nq, nc, cw, hc, n, K, eps, dil, want_s):
    """kv [T, hc*n + n], gate, s, normed and out of the block (the kernels)."""
    T = emb.shape[0]
    H = hist.shape[0]
    dev = emb.device
    lib = L.load()
    stream = L.stream_of(dev)
    kv = project(emb, w, torch.empty(T, hc * n + n, device=dev))
    stride = hc * n + n
    value = kv[:, hc * n:]
    gate = torch.empty(T, hc, device=dev)
    s = torch.empty(T, hc, device=dev) if want_s else None
    normed = torch.empty(T, hc, n, device=dev)
    st = lib.engram_ple_gate(kv.data_ptr(), stride, value.data_ptr(), stride, hidden.data_ptr(), nk.data_ptr(),
                             nq.data_ptr(), nc.data_ptr(), T, hc, n, eps, gate.data_ptr(), L.ptr(s),
                             normed.data_ptr(), stream)
    L.check(st, "engram_ple_gate")
    out = torch.empty(T, hc, n, device=dev)
    st = lib.engram_ple_conv(value.data_ptr(), stride, hidden.data_ptr(), gate.data_ptr(), normed.data_ptr(),
                             hist.data_ptr() if H else None, H, cw.data_ptr(), K, dil, T, hc, n, out.data_ptr(),
                             stream)
    L.check(st, "engram_ple_conv")
    return kv, gate, s, normed, out


class _PleBlockFn(torch.autograd.Function):
    """The block with gradients of emb, hidden and hist (weights frozen)."""

    @staticmethod
    def forward(ctx, emb, hidden, hist, w, nk, nq, nc, cw, meta):
        hc, n, K, eps, dil, detach_value, detach_gate = meta
        kv, gate, s, normed, out = _block_forward(emb, hidden, w, hist, nk, nq, nc, cw, hc, n, K, eps, dil, True)
        hist_len = (K - 1) * dil
        full = torch.cat([hist, normed], dim=0) if hist.shape[0] else normed
        new_hist = full[-hist_len:].clone() if hist_len > 0 else full[:0].clone()
        ctx.save_for_backward(hidden, hist, kv, gate, s, normed, nk, nq, nc, cw)
        ctx.w, ctx.meta = w, meta
        ctx.tail_len = new_hist.shape[0]
        ctx.mark_non_differentiable(gate, s)
        return out, new_hist, gate, s

    @staticmethod
    def backward(ctx, dout, dtail, _dgate, _ds):
        hidden, hist, kv, gate, s, normed, nk, nq, nc, cw = ctx.saved_tensors
        hc, n, K, eps, dil, detach_value, detach_gate = ctx.meta
        T, H = hidden.shape[0], hist.shape[0]
        dev = hidden.device
        lib = L.load()
        stream = L.stream_of(dev)
        dout = torch.zeros_like(hidden) if dout is None else dout.contiguous()
        dtail = None if dtail is None or ctx.tail_len == 0 else dtail.contiguous()
        dconv = torch.empty(T, hc, n, device=dev)
        dnormed = torch.empty(T, hc, n, device=dev)
        dhist = torch.empty(H, hc, n, device=dev) if (H and ctx.needs_input_grad[2]) else None
        st = lib.engram_ple_conv_backward(normed.data_ptr(), hist.data_ptr() if H else None, H, cw.data_ptr(), K, dil,
                                          T, hc, n, dout.data_ptr(), L.ptr(dtail), ctx.tail_len if dtail is not None
                                          else 0, dconv.data_ptr(), dnormed.data_ptr(), L.ptr(dhist), stream)
        L.check(st, "engram_ple_conv_backward")
        stride = hc * n + n
        dkv = torch.empty(T, stride, device=dev)
        dhidden = torch.empty(T, hc, n, device=dev)
        st = lib.engram_ple_gate_backward(kv.data_ptr(), stride, kv[:, hc * n:].data_ptr(), stride, hidden.data_ptr(),
                                          nk.data_ptr(), nq.data_ptr(), nc.data_ptr(), gate.data_ptr(), s.data_ptr(),
                                          dout.data_ptr(), dnormed.data_ptr(), T, hc, n, eps, int(detach_value),
                                          int(detach_gate), dkv.data_ptr(), stride, dkv[:, hc * n:].data_ptr(), stride,
                                          dhidden.data_ptr(), stream)
        L.check(st, "engram_ple_gate_backward")
        demb = None
        if ctx.needs_input_grad[0]:
            demb = project_back(dkv, ctx.w, torch.empty(T, n, device=dev))
        return (demb, dhidden if ctx.needs_input_grad[1] else None, dhist, None, None, None, None, None, None)


def _f32(x: torch.Tensor, name: str, shape) -> torch.Tensor:
    if not x.is_cuda or x.dtype != torch.float32:
        raise ValueError(f"{name}: needs a float32 CUDA tensor (got {x.dtype} on {x.device})")
    if tuple(x.shape) != tuple(shape):
        raise ValueError(f"{name}: shape {tuple(x.shape)}, expected {tuple(shape)}")
    return x.contiguous()


def ple_forward(emb: torch.Tensor, hidden: torch.Tensor, w, hist: torch.Tensor, hparams,
                diag: dict | None = None, detach_value: bool = False, detach_gate: bool = False):
    """(hidden + gated + silu(conv), new history tail): see the reference's
    docstring.  Differentiable in emb, hidden and hist (detach_value /
    detach_gate as in the reference); diag receives the same five tensors."""
    if weights_need_grad(w):
        raise NotImplementedError("engraft_ngram_b200.ple_forward does not build gradients of the block's weights; "
                                  "install_ple routes such calls to the reference's ple_forward")
    hc, n = int(hparams.hc_mult), int(hparams.n_embd)
    eps, dil = float(hparams.f_norm_rms_eps), int(hparams.ple_ngram_size)
    T = emb.shape[0]
    K = int(w.conv1d.shape[1])
    emb = _f32(emb, "emb", (T, n))
    hidden = _f32(hidden, "hidden", (T, hc, n))
    _f32(w.w_key, "w_key", (hc * n, n))
    _f32(w.w_value, "w_value", (n, n))
    nk = _f32(w.norm_key.detach().reshape(-1), "norm_key", (hc * n,))
    nq = _f32(w.norm_query.detach().reshape(-1), "norm_query", (hc * n,))
    nc = _f32(w.norm_conv.detach().reshape(-1), "norm_conv", (hc * n,))
    cw = _f32(w.conv1d.detach(), "conv1d", (hc * n, K))
    H = hist.shape[0]
    hist = _f32(hist, "hist", (H, hc, n)) if H else hist.reshape(0, hc, n)
    if needs_grad(emb, hidden, w, hist):
        out, new_hist, gate, s = _PleBlockFn.apply(emb, hidden, hist, w, nk, nq, nc, cw,
                                                   (hc, n, K, eps, dil, bool(detach_value), bool(detach_gate)))
        value = None
    else:
        kv, gate, s, normed, out = _block_forward(emb, hidden, w, hist, nk, nq, nc, cw, hc, n, K, eps, dil,
                                                  diag is not None)
        value = kv[:, hc * n:]
        hist_len = (K - 1) * dil
        hist_full = torch.cat([hist.to(normed.dtype), normed], dim=0) if H else normed
        new_hist = hist_full[-hist_len:] if hist_len > 0 else hist_full[:0]
    if diag is not None:
        with torch.no_grad():
            if value is None:  # the differentiable call keeps no value: project again for the diagnostics
                value = project(emb.detach(), w, torch.empty(T, hc * n + n, device=emb.device))[:, hc * n:]
            diag["s"] = s.detach().clone()
            diag["gate"] = gate.detach().clone()
            diag["value_norm"] = value.norm(dim=-1)
            diag["gated_norm"] = (value.unsqueeze(1) * gate.detach().unsqueeze(-1)).norm(dim=-1)
            diag["hidden_norm"] = hidden.detach().norm(dim=-1)
    return out, new_hist
