"""Pins the CPU oracle to the reference: every function is checked against the
golden vectors that tests/golden/make_golden.py produced by running the
reference (fulvian/engraft-ngram) itself."""
from __future__ import annotations

import numpy as np
import pytest

import fixtures as FX
from cases import fake_table, overlay_case, sha, syn_table
from oracle import oracle as O


def test_hash_fake_table_matches_reference(golden):
    # engraft/testing/fake_table.py:41-66 on the damage-test corpus shape
    p = FX.fake_table_params(seed=7)
    ids = O.hash_ids(golden["hash_fake_tokens"], p["ngram_size"], p["hpn"], p["mult"], p["head_sizes"],
                     p["head_offsets"], p["eos"])
    assert np.array_equal(ids, golden["hash_fake_ids"])


def test_hash_synthetic_pletable_matches_reference(golden):
    # engraft/table.py:111-144 through the real PleTable reader on a GGUF
    t = syn_table()
    assert np.array_equal(t.ids(golden["hash_syn_tokens"]), golden["hash_syn_ids"])


@pytest.mark.parametrize("k", range(9))
def test_hash_edge_cases_match_reference(golden, k):
    t = syn_table()
    toks = golden[f"edge{k}_tokens"]
    assert np.array_equal(t.ids(toks), golden[f"edge{k}_ids"].reshape(-1, 16))


def test_dequant_iq4nl_bit_exact(golden):
    got = O.dequant(O.FMT_IQ4_NL, 160, golden["dq_nl_raw"])
    assert np.array_equal(got.view(np.uint32), golden["dq_nl_out"].view(np.uint32))


def test_dequant_iq4xs_bit_exact(golden):
    got = O.dequant(O.FMT_IQ4_XS, 256, golden["dq_xs_raw"])
    assert np.array_equal(got.view(np.uint32), golden["dq_xs_out"].view(np.uint32))


def _run_overlay(c):
    ids = c.table.ids(c.tokens, seg_start=c.seg_start, t0=c.t0, n=c.n)
    emb, slots = O.forward(c.table.fmt, c.table.dim, c.table.raw, ids, 8, c.rows_init, c.row_ids)
    grad_rows = O.backward(slots, 8, c.grad, c.table.dim, len(c.row_ids))
    return emb, slots, grad_rows


@pytest.mark.parametrize("prefix", ["ov_syn_", "ov_synnoseg_"])
def test_overlay_forward_backward_iq4nl_bit_exact(golden, prefix):
    c = overlay_case(golden, prefix, syn_table())
    emb, slots, grad_rows = _run_overlay(c)
    assert sha(emb) == str(c.golden["emb_sha"])
    assert int((slots >= 0).sum()) == int(c.golden["n_id_hits"])
    assert np.array_equal(grad_rows.view(np.uint32), c.golden["grad_rows"].view(np.uint32))


def test_overlay_forward_backward_fake_table_bit_exact(golden, fake1_rows):
    c = overlay_case(golden, "ov_fake_", fake_table(fake1_rows, seed=1))
    emb, slots, grad_rows = _run_overlay(c)
    assert sha(emb) == str(c.golden["emb_sha"])
    assert int((slots >= 0).sum()) == int(c.golden["n_id_hits"])
    assert np.array_equal(grad_rows.view(np.uint32), c.golden["grad_rows"].view(np.uint32))


def test_backward_order_independent_of_threads(golden):
    c = overlay_case(golden, "ov_syn_", syn_table())
    n0 = O.num_threads()
    try:
        O.set_num_threads(1)
        a = _run_overlay(c)[2]
        O.set_num_threads(max(3, n0))
        b = _run_overlay(c)[2]
    finally:
        O.set_num_threads(n0)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_adam_with_regulariser_matches_torch_adam(golden):
    # engraft/descend_corpus.py:921-947 with torch.optim.Adam defaults
    rows0 = golden["adam_rows0"]
    p = rows0.copy()
    m = np.zeros_like(p)
    v = np.zeros_like(p)
    rs = np.float32(np.float32(golden["adam_mu"]) / golden["adam_S"])
    for k in range(golden["adam_grads"].shape[0]):
        O.adam_(p, golden["adam_grads"][k], m, v, k + 1, float(golden["adam_lr"]), p0=rows0, reg_scale=rs)
        norm = np.linalg.norm(golden["adam_traj"][k], axis=1, keepdims=True)
        err = np.abs(p - golden["adam_traj"][k])
        assert (err <= 1e-6 * norm).all(), float((err / norm).max())
        assert np.allclose(m, golden["adam_m"][k], rtol=1e-5, atol=1e-12)
        assert np.allclose(v, golden["adam_v"][k], rtol=1e-5, atol=1e-15)


def test_pack_layouts_roundtrip(golden):
    # the resident layouts hold the same bytes as the reference rows
    raw = golden["dq_nl_raw"]
    pk = O.pack(O.FMT_IQ4_NL, 160, raw)
    assert pk.shape == (64, 96)
    assert np.array_equal(pk[:, :80].reshape(64, 5, 16), raw.reshape(64, 5, 18)[:, :, 2:])
    assert np.array_equal(pk[:, 80:90].reshape(64, 5, 2), raw.reshape(64, 5, 18)[:, :, :2])
    xs = golden["dq_xs_raw"]
    pk = O.pack(O.FMT_IQ4_XS, 256, xs)
    assert pk.shape == (48, 144)
    assert np.array_equal(pk[:, :128], xs[:, 8:]) and np.array_equal(pk[:, 128:136], xs[:, :8])


def test_scan_hits_matches_reference(golden):
    # engraft/damage.py:168-224 on the reference's own test corpus shape
    p = FX.fake_table_params(seed=7)
    got = O.scan_hits(golden["scan_tokens"], p["ngram_size"], p["hpn"], p["mult"], p["head_sizes"],
                      p["head_offsets"], p["eos"], golden["scan_overlay"], golden["scan_dnorm"])
    assert np.array_equal(got["pos"], golden["scan_pos"])
    assert np.array_equal(got["n_hit_rows"], golden["scan_n_hit_rows"])
    assert np.array_equal(got["dnorm_max"].view(np.uint32), golden["scan_dnorm_max"].view(np.uint32))
    assert np.array_equal(got["dnorm_sum"].view(np.uint32), golden["scan_dnorm_sum"].view(np.uint32))
    assert np.array_equal(got["read_count"], golden["scan_read_count"])


# ---------------------------------------------------------------- row sets
def _fake7():
    p = FX.fake_table_params(seed=7)
    return p, (3, 8, p["mult"], p["head_sizes"], p["head_offsets"], p["eos"])


def test_oracle_rows_read_by_prefixes_matches_reference_golden(golden):
    p, geo = _fake7()
    frags = FX.fragments(seed=31, n_frag=12, vocab=50, eos=p["eos"], lo=3, hi=120)
    got = O.rows_read_by_prefixes(frags, *geo)
    assert np.array_equal(got, golden["rowset_all_read"])


@pytest.mark.parametrize("policy", ["all-read", "private", "entity", "t8-answer"])
def test_oracle_rows_var_ids_match_reference_golden(golden, policy):
    p, geo = _fake7()
    frags = FX.fragments(seed=31, n_frag=12, vocab=50, eos=p["eos"], lo=3, hi=120)
    sets = FX.rowset_case_sets(golden["rowset_all_read"])
    got = O.rows_var_ids(policy, sets, frags, FX.ROWSET_EXCLUDE, *geo)
    assert np.array_equal(got, golden[f"rowset_{policy.replace('-', '_')}_ids"])


def test_oracle_sum_overlays_matches_reference_golden(golden):
    import ast
    import hashlib
    rows7 = FX.fake_table_rows(seed=7)
    all_read = golden["rowset_all_read"]
    files = [FX.pleo_fact(k, all_read, rows7[all_read]) for k in range(3)]
    union, merged, (moved, shared, hist) = O.sum_overlays(files, lambda ids: rows7[np.asarray(ids)])
    assert np.array_equal(union, golden["sumov_union"])
    assert hashlib.sha256(merged.tobytes()).hexdigest() == str(golden["sumov_merged_sha"])
    man = ast.literal_eval(str(golden["sumov_manifest"]))
    assert (moved, shared, hist) == (man["n_rows_moved_any"], man["n_rows_shared"], man["facts_per_row_histogram"])


PLE_TOL = 2e-6  # fp32: numpy's and torch's reductions and matmuls round in different orders


@pytest.mark.parametrize("case", FX.PLE_CASES)
def test_ple_block_oracle_matches_reference(golden, case):
    """The numpy restatement of ple_forward against the reference's own torch
    function on the same seeded inputs (empty, full, single-step and short
    histories): output and new history within PLE_TOL relative to the largest
    magnitude."""
    seed, T, n_hist = case
    c = FX.ple_case(seed, T, n_hist)
    out, hist = O.ple_forward(c["emb"], c["hidden"], c["w_key"], c["w_value"], c["norm_key"], c["norm_query"],
                              c["norm_conv"], c["conv1d"], c["hist"], FX.PLE_HC, FX.PLE_N, FX.PLE_EPS, FX.PLE_DIL)
    ref_out, ref_hist = golden[f"ple{seed}_out"], golden[f"ple{seed}_hist"]
    assert out.shape == ref_out.shape and hist.shape == ref_hist.shape
    assert np.abs(out - ref_out).max() <= PLE_TOL * max(1.0, np.abs(ref_out).max())
    assert np.abs(hist - ref_hist).max() <= PLE_TOL * max(1.0, np.abs(ref_hist).max())


def test_ple_backward_restatement_matches_reference_golden():
    """The float64 torch restatement of the PLE block (cases.ple_block_torch),
    differentiated by autograd, gives the reference's own gradients of emb,
    hidden and hist (tests/golden/ple_backward_golden.npz, made by running the
    reference), with the detach_value / detach_gate variants."""
    import torch
    import fixtures as FX
    from cases import ple_block_torch
    from make_ple_backward_golden import VARIANTS, upstream
    from pathlib import Path
    gold = np.load(Path(__file__).parent / "golden" / "ple_backward_golden.npz")
    for idx, (seed, T, n_hist) in enumerate(FX.PLE_CASES):
        c = FX.ple_case(seed, T, n_hist)
        w = {k: torch.from_numpy(c[k]).double() for k in
             ("w_key", "w_value", "norm_key", "norm_query", "norm_conv", "conv1d")}
        for suffix, dv, dg in (VARIANTS if idx == 0 else VARIANTS[:1]):
            emb, hidden, hist = (torch.from_numpy(c[k]).double().requires_grad_(True) for k in ("emb", "hidden", "hist"))
            o, h = ple_block_torch(emb, hidden, w, hist, FX.PLE_HC, FX.PLE_N, FX.PLE_EPS, FX.PLE_DIL, dv, dg)
            dout, dtail = upstream(seed, T, h.shape[0])
            ((o * torch.from_numpy(dout).double()).sum() + (h * torch.from_numpy(dtail).double()).sum()).backward()
            for name, t in (("demb", emb), ("dhidden", hidden), ("dhist", hist)):
                want = gold[f"ple{seed}{suffix}_{name}"]
                got = t.grad.numpy() if t.grad is not None else np.zeros_like(want)
                assert got.shape == want.shape
                assert want.size == 0 or np.abs(got - want).max() <= 1e-5 * max(1.0, np.abs(want).max()), (seed, suffix, name)
