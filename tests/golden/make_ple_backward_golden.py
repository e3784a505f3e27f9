"""Generates tests/golden/ple_backward_golden.npz by running the REFERENCE's own
PLE block (engraft/replica/layers.py:565-626, ple_forward) with torch autograd
on the seeded cases of fixtures.PLE_CASES: the gradients of emb, hidden and
hist for a seeded upstream gradient of out and of the new history tail, and,
on the first case, with the reference's detach_value / detach_gate flags.

    python tests/golden/make_ple_backward_golden.py /path/to/engraft-ngram

Only the .npz it writes is used at test time.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import fixtures as FX  # noqa: E402

VARIANTS = [("", False, False), ("dv", True, False), ("dg", False, True)]  # name suffix, detach_value, detach_gate


def upstream(seed: int, T: int, tail: int):
    """The seeded upstream gradients of one case: of out [T, hc, n] and of the
    new history tail [tail, hc, n]."""
    rng = np.random.default_rng(5000 + seed)
    dout = rng.standard_normal((T, FX.PLE_HC, FX.PLE_N)).astype(np.float32)
    dtail = rng.standard_normal((tail, FX.PLE_HC, FX.PLE_N)).astype(np.float32)
    return dout, dtail


def main(ref_root: str) -> None:
    sys.path.insert(0, str(Path(ref_root).resolve()))
    import torch
    import engraft.replica.layers as RL
    torch.set_num_threads(1)

    class _PleHP:
        hc_mult, n_embd, f_norm_rms_eps, ple_ngram_size = FX.PLE_HC, FX.PLE_N, FX.PLE_EPS, FX.PLE_DIL

    out = {}
    for idx, (seed, T, n_hist) in enumerate(FX.PLE_CASES):
        c = FX.ple_case(seed, T, n_hist)
        w = RL.PleWeights(**{k: torch.from_numpy(c[k]) for k in
                             ("w_key", "w_value", "norm_key", "norm_query", "norm_conv", "conv1d")})
        for suffix, dv, dg in (VARIANTS if idx == 0 else VARIANTS[:1]):
            emb = torch.from_numpy(c["emb"]).requires_grad_(True)
            hidden = torch.from_numpy(c["hidden"]).requires_grad_(True)
            hist = torch.from_numpy(c["hist"]).requires_grad_(True)
            o, h = RL.ple_forward(emb, hidden, w, hist, _PleHP, detach_value=dv, detach_gate=dg)
            dout, dtail = upstream(seed, T, h.shape[0])
            loss = (o * torch.from_numpy(dout)).sum() + (h * torch.from_numpy(dtail)).sum()
            loss.backward()
            key = f"ple{seed}{suffix}"
            out[f"{key}_demb"] = emb.grad.numpy()
            out[f"{key}_dhidden"] = hidden.grad.numpy()
            out[f"{key}_dhist"] = (hist.grad.numpy() if hist.grad is not None
                                   else np.zeros_like(c["hist"]))
    out["meta"] = np.array(repr(dict(reference_root=str(ref_root), torch=torch.__version__)))
    dst = HERE / "ple_backward_golden.npz"
    np.savez_compressed(dst, **out)
    print(f"wrote {dst} ({dst.stat().st_size} bytes, {len(out)} arrays)")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/make_ple_backward_golden.py <path of the reference checkout>")
    main(sys.argv[1])
