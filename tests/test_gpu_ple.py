"""The PLE block (engraft/replica/layers.py:565-626) on the GPU against the
reference's own outputs (golden vectors), the numpy oracle and, at the real
width (hc = 4, n_embd = 2560), a plain torch fp32 statement of the same
formula."""
from __future__ import annotations

import types

import numpy as np
import pytest
import torch

import fixtures as FX
from oracle import oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
TOL = 2e-5  # fp32, relative to the largest magnitude: cuBLAS and the block reductions round in their own order


def _weights(c):
    return types.SimpleNamespace(**{k: torch.from_numpy(c[k]).to(DEV) for k in
                                    ("w_key", "w_value", "norm_key", "norm_query", "norm_conv", "conv1d")})


def _hp(hc, n, dil=FX.PLE_DIL, eps=FX.PLE_EPS):
    return types.SimpleNamespace(hc_mult=hc, n_embd=n, f_norm_rms_eps=eps, ple_ngram_size=dil)


def _close(got, want):
    got = got.detach().cpu().numpy() if isinstance(got, torch.Tensor) else got
    return np.abs(got - want).max() <= TOL * max(1.0, np.abs(want).max())


@pytest.fixture(params=["3xtf32", "fp32", "tcgen05"])
def projection(request, monkeypatch):
    from engraft_ngram_b200 import ple
    monkeypatch.setattr(ple, "PROJECTION", request.param)
    return request.param


@pytest.mark.parametrize("case", FX.PLE_CASES)
def test_ple_block_matches_reference_golden(golden, case, projection):
    import engraft_ngram_b200 as eb
    seed, T, n_hist = case
    c = FX.ple_case(seed, T, n_hist)
    d = {}
    out, hist = eb.ple_forward(torch.from_numpy(c["emb"]).to(DEV), torch.from_numpy(c["hidden"]).to(DEV),
                               _weights(c), torch.from_numpy(c["hist"]).to(DEV), _hp(FX.PLE_HC, FX.PLE_N), diag=d)
    torch.cuda.synchronize()
    ref_out, ref_hist = O.ple_forward(c["emb"], c["hidden"], c["w_key"], c["w_value"], c["norm_key"],
                                      c["norm_query"], c["norm_conv"], c["conv1d"], c["hist"], FX.PLE_HC, FX.PLE_N,
                                      FX.PLE_EPS, FX.PLE_DIL)
    assert _close(out, ref_out) and _close(hist, ref_hist)
    assert _close(out, golden[f"ple{seed}_out"]) and _close(hist, golden[f"ple{seed}_hist"])
    assert set(d) == {"s", "gate", "value_norm", "gated_norm", "hidden_norm"} and d["gate"].shape == (T, FX.PLE_HC)


def _torch_ple(emb, hidden, w, hist, hc, n, eps, dil):
    """The reference formula in plain torch fp32 on the GPU (TF32 off)."""
    T = emb.shape[0]

    def rms(x, wt):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * wt.reshape(hc, n)

    key = (emb @ w.w_key.T).reshape(T, hc, n)
    s = (rms(key, w.norm_key) * rms(hidden, w.norm_query)).sum(-1) / n ** 0.5
    gate = torch.sigmoid(torch.sign(s) * torch.sqrt(s.abs().clamp_min(1e-6)))
    value = emb @ w.w_value.T
    gated = value.unsqueeze(1) * gate.unsqueeze(-1)
    normed = rms(gated, w.norm_conv)
    K = w.conv1d.shape[1]
    full = torch.cat([hist, normed]).reshape(-1, hc * n)
    H = hist.shape[0]
    acc = torch.zeros(T, hc * n, device=emb.device)
    for k in range(K):
        back = (K - 1 - k) * dil
        for t in range(T):
            if H + t - back >= 0:
                acc[t] += full[H + t - back] * w.conv1d[:, k]
    out = hidden + gated + torch.nn.functional.silu(acc).reshape(T, hc, n)
    return out, torch.cat([hist, normed])[-(K - 1) * dil:]


@pytest.mark.parametrize("T,n_hist", [(6, 9), (24, 0)])
def test_ple_block_at_real_width(T, n_hist, projection):
    """hc = 4, n_embd = 2560, K = 4, dilation 3 (the reference's PLE layer)."""
    import engraft_ngram_b200 as eb
    hc, n, K = 4, 2560, 4
    g = torch.Generator(device=DEV).manual_seed(T)
    r = lambda *s: torch.randn(*s, generator=g, device=DEV) * 0.1  # noqa: E731
    w = types.SimpleNamespace(w_key=r(hc * n, n), w_value=r(n, n), norm_key=1 + r(hc * n), norm_query=1 + r(hc * n),
                              norm_conv=1 + r(hc * n), conv1d=r(hc * n, K))
    emb, hidden, hist = r(T, n), r(T, hc, n), r(n_hist, hc, n)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        want_out, want_hist = _torch_ple(emb, hidden, w, hist, hc, n, 1e-6, 3)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    out, new_hist = eb.ple_forward(emb, hidden, w, hist, _hp(hc, n, 3, 1e-6))
    torch.cuda.synchronize()
    assert _close(out, want_out.cpu().numpy()) and _close(new_hist, want_hist.cpu().numpy())


def _ple_grads(eb, c, hc, n, dout, dtail, dv=False, dg=False, w=None):
    emb, hidden, hist = (torch.as_tensor(c[k]).to(DEV).requires_grad_(True) for k in ("emb", "hidden", "hist"))
    w = w if w is not None else _weights(c)
    out, new_hist = eb.ple_forward(emb, hidden, w, hist, _hp(hc, n), detach_value=dv, detach_gate=dg)
    loss = (out * torch.as_tensor(dout).to(DEV)).sum() + (new_hist * torch.as_tensor(dtail).to(DEV)).sum()
    loss.backward()
    torch.cuda.synchronize()
    return {"demb": emb.grad, "dhidden": hidden.grad, "dhist": hist.grad}


@pytest.mark.parametrize("case", FX.PLE_CASES)
def test_ple_backward_matches_reference_golden(case, projection):
    """Gradients of emb, hidden and hist through the B200 block (the CUDA
    backward kernels and the projection GEMM back) equal the reference's own
    autograd gradients (tests/golden/ple_backward_golden.npz) within the fp32
    tolerance, with the detach_value / detach_gate variants on the first case."""
    from pathlib import Path
    import engraft_ngram_b200 as eb
    from make_ple_backward_golden import VARIANTS, upstream
    gold = np.load(Path(__file__).parent / "golden" / "ple_backward_golden.npz")
    seed, T, n_hist = case
    c = FX.ple_case(seed, T, n_hist)
    first = case == FX.PLE_CASES[0]
    for suffix, dv, dg in (VARIANTS if first else VARIANTS[:1]):
        tail = min((FX.PLE_K - 1) * FX.PLE_DIL, n_hist + T)
        dout, dtail = upstream(seed, T, tail)
        got = _ple_grads(eb, c, FX.PLE_HC, FX.PLE_N, dout, dtail, dv, dg)
        for name in ("demb", "dhidden", "dhist"):
            want = gold[f"ple{seed}{suffix}_{name}"]
            g = got[name]
            if want.size == 0:
                continue
            assert g is not None and _close(g, want), (seed, suffix, name)


@pytest.mark.parametrize("T,n_hist", [(24, 0), (6, 9)])
def test_ple_backward_at_real_width(T, n_hist, projection):
    """hc = 4, n_embd = 2560, K = 4, dilation 3: the CUDA backward against the
    float64 torch restatement of the block differentiated by autograd."""
    import engraft_ngram_b200 as eb
    from cases import ple_block_torch
    hc, n, K = 4, 2560, 4
    g = torch.Generator(device=DEV).manual_seed(100 + T)
    r = lambda *s: torch.randn(*s, generator=g, device=DEV) * 0.1  # noqa: E731
    wd = dict(w_key=r(hc * n, n), w_value=r(n, n), norm_key=1 + r(hc * n), norm_query=1 + r(hc * n),
              norm_conv=1 + r(hc * n), conv1d=r(hc * n, K))
    c = dict(emb=r(T, n), hidden=r(T, hc, n), hist=r(n_hist, hc, n))
    tail = min((K - 1) * 3, n_hist + T)
    dout, dtail = torch.randn(T, hc, n, generator=g, device=DEV), torch.randn(tail, hc, n, generator=g, device=DEV)
    got = _ple_grads(eb, c, hc, n, dout, dtail, w=types.SimpleNamespace(**wd))
    emb, hidden, hist = (c[k].double().requires_grad_(True) for k in ("emb", "hidden", "hist"))
    o, h = ple_block_torch(emb, hidden, {k: v.double() for k, v in wd.items()}, hist, hc, n, 1e-6, 3)
    ((o * dout.double()).sum() + (h * dtail.double()).sum()).backward()
    for name, t in (("demb", emb), ("dhidden", hidden), ("dhist", hist)):
        if t.grad is None or t.numel() == 0:
            continue
        assert _close(got[name], t.grad.float().cpu().numpy()), name


def test_ple_block_weight_gradients_route_to_the_reference():
    """Gradients of emb, hidden and hist run on the B200 block; a call that
    needs gradients of the block's weights raises there, and install_ple sends
    exactly those calls to the original function."""
    import engraft_ngram_b200 as eb
    c = FX.ple_case(1, 3, 0)
    w = _weights(c)
    emb = torch.from_numpy(c["emb"]).to(DEV).requires_grad_(True)
    hidden = torch.from_numpy(c["hidden"]).to(DEV)
    hist = torch.from_numpy(c["hist"]).to(DEV)
    out, _ = eb.ple_forward(emb, hidden, w, hist, _hp(FX.PLE_HC, FX.PLE_N))
    out.sum().backward()
    assert emb.grad is not None and torch.isfinite(emb.grad).all()
    w_train = _weights(c)
    w_train.conv1d.requires_grad_(True)
    with pytest.raises(NotImplementedError):
        eb.ple_forward(emb, hidden, w_train, hist, _hp(FX.PLE_HC, FX.PLE_N))
    calls = []
    fake = types.ModuleType("fake_layers")
    fake.ple_forward = lambda *a, **k: calls.append("orig") or ("orig", None)
    fake_model = types.ModuleType("fake_model")
    fake_model.ple_forward = fake.ple_forward
    mods = {"engraft.replica.layers": fake, "engraft.replica.model": fake_model}
    eb.install_ple(mods)
    try:
        assert fake.ple_forward(emb, hidden, w_train, hist, _hp(FX.PLE_HC, FX.PLE_N)) == ("orig", None)
        out, _ = fake_model.ple_forward(emb, hidden, w, hist, _hp(FX.PLE_HC, FX.PLE_N))  # emb needs a gradient
        assert isinstance(out, torch.Tensor) and out.requires_grad and calls == ["orig"]
    finally:
        eb.uninstall_ple(mods)
    assert fake.ple_forward is not None and fake.ple_forward(None, None, None, None, None) == ("orig", None)


@pytest.mark.parametrize("M,N,K,terms", [(128, 256, 32, 1), (11, 300, 36, 1), (256, 768, 256, 3),
                                         (2048, 2560, 1024, 3), (333, 513, 1000, 2)])
def test_tcgen05_gemm_matches_float64(M, N, K, terms):
    """engram_gemm_tf32 (tcgen05 MMAs, TMA-fed, TMEM accumulator): one TF32 term
    within TF32 rounding of the float64 product; the 3xTF32 split within fp32
    accumulation error; ragged M, N and K handled by the zero-filled tiles; no
    barrier wait gave up."""
    from engraft_ngram_b200.ple import gemm_tf32, split_tf32
    g = torch.Generator(device=DEV).manual_seed(M + N + K)
    A = torch.randn(M, K, generator=g, device=DEV)
    B = torch.randn(N, K, generator=g, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = torch.full((M, N), float("nan"), device=DEV)
    if terms == 1:
        gemm_tf32([(A, B)], out, err)
        tol = 4e-3
    else:
        a_hi, a_lo = split_tf32(A)
        b_hi, b_lo = split_tf32(B)
        gemm_tf32([(a_lo, b_hi), (a_hi, b_lo), (a_hi, b_hi)][-terms:], out, err)
        tol = 2e-5 if terms == 3 else 3e-3
    torch.cuda.synchronize()
    want = A.double() @ B.double().T
    assert int(err.item()) == 0
    assert torch.isfinite(out).all()
    rel = ((out.double() - want).abs().max() / want.abs().max()).item()
    assert rel <= tol, rel


@pytest.mark.parametrize("M,N,K", [(128, 256, 16), (11, 300, 36), (256, 768, 256), (2048, 2560, 1024),
                                   (333, 513, 1000)])
def test_fused_3xtf32_gemm_matches_float64_and_the_three_terms(M, N, K):
    """engram_gemm_3xtf32 (one load of A_hi, A_lo, B_hi, B_lo per K slice, three
    MMAs from it) is within fp32 accumulation error of the float64 product and
    agrees with engram_gemm_tf32 over the same three terms to accumulation
    order; ragged shapes zero-filled; no barrier wait gave up."""
    from engraft_ngram_b200.ple import gemm_3xtf32, gemm_tf32, split_tf32
    g = torch.Generator(device=DEV).manual_seed(3 * M + N + K)
    A = torch.randn(M, K, generator=g, device=DEV)
    B = torch.randn(N, K, generator=g, device=DEV)
    a_hi, a_lo = split_tf32(A)
    b_hi, b_lo = split_tf32(B)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    fused = torch.full((M, N), float("nan"), device=DEV)
    gemm_3xtf32(a_hi, a_lo, b_hi, b_lo, fused, err)
    terms = torch.full((M, N), float("nan"), device=DEV)
    gemm_tf32([(a_lo, b_hi), (a_hi, b_lo), (a_hi, b_hi)], terms, err)
    torch.cuda.synchronize()
    want = A.double() @ B.double().T
    scale = want.abs().max()
    assert int(err.item()) == 0
    assert torch.isfinite(fused).all()
    assert ((fused.double() - want).abs().max() / scale).item() <= 2e-5
    assert ((fused.double() - terms.double()).abs().max() / scale).item() <= 2e-5
