"""Generates the golden vectors in this folder by running the REFERENCE itself
(fulvian/engraft-ngram, imported from its source tree) on seeded inputs.

Run in a container that holds the reference source (it is not needed at test
time: only the .npz files it writes are committed):

    python tests/golden/make_golden.py /path/to/engraft-ngram

Every output that the reference computes exactly (row ids, dequantised rows,
the gathered embedding, the sequentially accumulated row gradients) is stored
so the tests can demand bit equality; the Adam trajectory is stored in full.
torch runs single-threaded here: with one thread, index_put_(accumulate=True)
adds duplicate rows serially in index order, the same order the reference's
CUDA path uses (stable sort), so the stored gradients are the canonical ones.
"""
from __future__ import annotations

import hashlib
import struct
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import fixtures as FX  # noqa: E402


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def write_syn_gguf(path: Path, gguf) -> None:
    """Per-head IQ4_NL table GGUF with the metadata PleTable reads
    (engraft/table.py:48-88)."""
    p = FX.syn_params()
    raw = FX.syn_table_raw()
    w = gguf.GGUFWriter(str(path), arch="qwen4exp")
    V = gguf.GGUFValueType
    w.add_uint32("qwen4exp.ple.eos_token_id", p["eos"])
    w.add_uint32("qwen4exp.ple.image_token_id", FX.SYN_IMAGE_TOKEN)
    w.add_uint32("qwen4exp.ple.ngram_size", p["ngram_size"])
    w.add_uint32("qwen4exp.ple.heads_per_ngram", p["hpn"])
    w.add_key_value("qwen4exp.ple.layer_multipliers", p["mult"], V.ARRAY, sub_type=V.UINT64)
    w.add_key_value("qwen4exp.ple.head_vocab_sizes", p["head_sizes"], V.ARRAY, sub_type=V.UINT32)
    w.add_key_value("qwen4exp.ple.head_offsets", p["head_offsets"], V.ARRAY, sub_type=V.UINT32)
    for h, (off, ph) in enumerate(zip(p["head_offsets"], p["head_sizes"])):
        w.add_tensor(f"ple_ngram_embd.{h}.weight", raw[off:off + ph], raw_dtype=gguf.GGMLQuantizationType.IQ4_NL)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


def _head_local(table, g: int) -> tuple[int, int]:
    """(head, local index) of global row g."""
    offs = np.asarray(table.head_offsets, dtype=np.int64)
    h = int(np.searchsorted(offs, g, side="right") - 1)
    return h, g - int(offs[h])


def hash_case(table, tokens: list[int], damage) -> np.ndarray:
    from engraft.lens import local_to_global
    addr = table.ngram_addresses(tokens)
    ids = np.array([[local_to_global(table, h, a[h]) for h in range(table.n_heads)] for a in addr],
                   dtype=np.int64).reshape(len(tokens), table.n_heads)
    if len(tokens):
        big, tri = damage.ngram_rows(np.asarray(tokens, dtype=np.int64), table)
        assert np.array_equal(np.concatenate([big, tri], axis=1), ids), "scalar and vectorised hash differ"
    return ids.astype(np.int32)


EDGE_TOKEN_LISTS = [
    [],
    [5],
    ["EOS"],
    ["EOS", 3],
    [3, "EOS", 4, 5],
    ["EOS", "EOS", "EOS", 7],
    [1, 2, 3, 4, 5],
    [0, 0, 0],
    [2**31 - 1, 2**30, 17, -1, 3],
]


def overlay_case(table, seq, distill, pack, torch, frags, eos, n_pick_every, seed, dim=160,
                 extra_ids=(), start=0, use_segments=True):
    packed = pack.pack_fragments(frags, eos, max_len=4096)[0]
    tokens = packed.tokens
    n_prefix = len(tokens) - 1
    seg = packed.segment_ids if use_segments else None
    # rows read by the batch, as the descent's census would list them
    from engraft.lens import RowSet
    read = set()
    seg_starts = FX.seg_starts(packed.segment_ids.tolist())
    for t in range(n_prefix):
        s = int(seg_starts[t]) if use_segments else 0
        rs = RowSet.from_position(table, tokens[s:], t - s)
        read.update(int(g) for g in rs.rows_global)
    read = sorted(read)
    chosen = sorted(set(read[::n_pick_every]) | set(int(x) for x in extra_ids))
    row_map = {g: i for i, g in enumerate(chosen)}
    true_rows = distill._read_true_rows(table, chosen)
    rows_init = (true_rows + FX.overlay_noise(seed, true_rows.shape)).astype(np.float32)
    rows_var = torch.from_numpy(rows_init.copy()).requires_grad_(True)
    ov = seq.OverlayEmb(table, tokens, rows_var, row_map, segment_ids=seg)
    emb = ov.build(n_prefix, start=start)
    grad = torch.from_numpy(FX.overlay_grad(seed, tuple(emb.shape)))
    emb.backward(grad)
    return dict(
        tokens=np.asarray(tokens, dtype=np.int32),
        segment_ids=packed.segment_ids.numpy().astype(np.int32),
        use_segments=np.int32(1 if use_segments else 0),
        start=np.int32(start),
        n_prefix=np.int32(n_prefix),
        row_ids=np.asarray(chosen, dtype=np.int32),
        seed=np.int32(seed),
        rows_init_sha=sha(rows_init),
        emb_sha=sha(emb.detach().numpy()),
        emb_row1=emb.detach().numpy()[1].copy(),
        grad_rows=rows_var.grad.numpy().copy(),
        n_id_hits=np.int32(ov.n_id_hits),
    )


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    import gguf
    import torch
    torch.set_num_threads(1)
    import engraft.damage as damage
    import engraft.replica.distill as distill
    import engraft.replica.pack as pack
    import engraft.replica.seq as seq
    from engraft.lens import write_pleo
    from engraft.replica.dequant import dequant_iq4_xs
    from engraft.table import PleTable, dequant_iq4nl
    from engraft.testing.fake_table import FakeTable

    out = {}

    # ---- 1. hash: FakeTable(seed=7) over the damage-test corpus shape -------
    ft = FakeTable(seed=7)
    fp = FX.fake_table_params(seed=7)
    assert fp["mult"] == ft.layer_multipliers and fp["head_offsets"] == ft.head_offsets
    toks = FX.synthetic_corpus(1200, seed=1, eos=ft.eos_token_id)
    out["hash_fake_tokens"] = toks
    out["hash_fake_ids"] = hash_case(ft, toks.tolist(), damage)

    # ---- 2. hash + dequant + overlay on the synthetic IQ4_NL GGUF (real PleTable)
    with tempfile.TemporaryDirectory() as td:
        path = Path(td) / "syn_table.gguf"
        write_syn_gguf(path, gguf)
        table = PleTable(path)
        sp = FX.syn_params()
        assert table.layer_multipliers == sp["mult"] and table.head_vocab_sizes == sp["head_sizes"]
        assert table.eos_token_id == sp["eos"]
        rng = np.random.default_rng(3)
        toks = rng.integers(0, 248320, size=1000).astype(np.int64)
        toks[rng.integers(0, 1000, size=25)] = sp["eos"]
        toks[500:503] = sp["eos"]
        out["hash_syn_tokens"] = toks.astype(np.int32)
        out["hash_syn_ids"] = hash_case(table, toks.tolist(), damage)
        for k, lst in enumerate(EDGE_TOKEN_LISTS):
            tl = [sp["eos"] if x == "EOS" else int(x) for x in lst]
            out[f"edge{k}_tokens"] = np.asarray(tl, dtype=np.int32)
            out[f"edge{k}_ids"] = hash_case(table, tl, damage) if tl else np.zeros((0, 16), np.int32)
        # dequant of whole heads through the reader's stripe path vs gguf
        raw_h3 = table.read_rows_raw(3, 0, 64)
        out["dq_nl_raw"] = raw_h3
        out["dq_nl_out"] = dequant_iq4nl(raw_h3)
        ref = np.stack([gguf.quants.dequantize(raw_h3[i], gguf.GGMLQuantizationType.IQ4_NL).reshape(-1)
                        for i in range(raw_h3.shape[0])])
        assert np.array_equal(ref.view(np.uint32), out["dq_nl_out"].view(np.uint32))

        frags = FX.fragments(seed=11, n_frag=5, vocab=248320, eos=sp["eos"])
        case = overlay_case(table, seq, distill, pack, torch, frags, sp["eos"], n_pick_every=7, seed=5,
                            extra_ids=[0, 17, sum(FX.SYN_HEAD_SIZES) - 1])
        for k, v in case.items():
            out[f"ov_syn_{k}"] = v
        case = overlay_case(table, seq, distill, pack, torch, frags, sp["eos"], n_pick_every=9, seed=6,
                            use_segments=False, start=7)
        for k, v in case.items():
            out[f"ov_synnoseg_{k}"] = v

    # ---- 3. IQ4_XS dequant (model-weight format used for the 256-wide table)
    xs = FX.iq4xs_raw(48, seed=9)
    out["dq_xs_raw"] = xs
    got = dequant_iq4_xs(torch.from_numpy(xs)).numpy()
    ref = np.stack([gguf.quants.dequantize(xs[i], gguf.GGMLQuantizationType.IQ4_XS).reshape(-1)
                    for i in range(xs.shape[0])])
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    out["dq_xs_out"] = got

    # ---- 4. overlay on the fp32 FakeTable (the reference's own test fixture)
    ft1 = FakeTable(seed=1)
    frags = FX.fragments(seed=12, n_frag=4, vocab=60, eos=ft1.eos_token_id)
    case = overlay_case(ft1, seq, distill, pack, torch, frags, ft1.eos_token_id, n_pick_every=8, seed=7)
    for k, v in case.items():
        out[f"ov_fake_{k}"] = v

    # ---- 5. optimizer: descend_corpus.py:776-790 and :921-947 --------------
    R = 16
    rng = np.random.default_rng(21)
    rows0_np = FX.iq4nl_raw(R, seed=22)
    rows0_np = dequant_iq4nl(rows0_np)
    rows0 = torch.from_numpy(rows0_np.copy())
    rows_var = rows0.clone().detach().requires_grad_(True)
    mu, lr_scale = 0.10172, 4.9597
    mean_row_norm = float(rows0.norm(dim=1).mean().item())
    lr = lr_scale * 0.01 * mean_row_norm / (160 ** 0.5)
    opt = torch.optim.Adam([rows_var], lr=lr)
    grads = (rng.standard_normal((3, R, 160)) * 1e-3).astype(np.float32)
    grads[:, ::5] = 0.0  # rows the batch did not touch: moved only by the regulariser
    traj, msaved, vsaved = [], [], []
    for k in range(grads.shape[0]):
        opt.zero_grad()
        rows_var.grad = torch.from_numpy(grads[k].copy())
        reg = mu * ((rows_var - rows0).pow(2).sum() / rows0.pow(2).sum().clamp_min(1e-12))
        reg.backward()
        opt.step()
        st = opt.state[rows_var]
        traj.append(rows_var.detach().numpy().copy())
        msaved.append(st["exp_avg"].numpy().copy())
        vsaved.append(st["exp_avg_sq"].numpy().copy())
    out["adam_rows0"] = rows0_np
    out["adam_grads"] = grads
    out["adam_mu"] = np.float64(mu)
    out["adam_lr"] = np.float64(lr)
    out["adam_S"] = np.float32(rows0.pow(2).sum().clamp_min(1e-12).item())
    out["adam_traj"] = np.stack(traj)
    out["adam_m"] = np.stack(msaved)
    out["adam_v"] = np.stack(vsaved)

    # ---- 6. .pleo bytes (engraft/lens.py:33-46) -----------------------------
    with tempfile.TemporaryDirectory() as td:
        pth = Path(td) / "x.pleo"
        rows = np.array([5, 17, 319989556], dtype=np.int32)
        data = (np.arange(3 * 160, dtype=np.float32).reshape(3, 160) * 0.25 - 7.0).astype(np.float32)
        write_pleo(pth, rows, data)
        out["pleo_rows"] = rows
        out["pleo_data"] = data
        out["pleo_bytes"] = np.frombuffer(pth.read_bytes(), dtype=np.uint8).copy()

    # ---- 7. bulk hash + overlay hit scan (engraft/damage.py:168-224) -------
    ft7 = FakeTable(seed=7)
    toks = FX.synthetic_corpus(20_000, seed=1, eos=ft7.eos_token_id)
    big, tri = damage.ngram_rows(toks, ft7)
    rows16 = np.concatenate([big, tri], axis=1)
    rng = np.random.default_rng(77)
    picks = rows16[rng.integers(0, 19_999, size=60), rng.integers(0, 16, size=60)]
    overlay_sorted = np.unique(np.concatenate([picks, rng.integers(0, 80_000, size=40)])).astype(np.int32)
    dnorm_sorted = (rng.random(len(overlay_sorted)) * 0.3).astype(np.float32)
    dnorm_sorted[::7] = 0.0  # unchanged rows
    hits = damage.scan_hits(toks, ft7, overlay_sorted, dnorm_sorted, block=4_000)
    out["scan_tokens"] = toks
    out["scan_overlay"] = overlay_sorted
    out["scan_dnorm"] = dnorm_sorted
    for k in ("pos", "n_hit_rows", "dnorm_max", "dnorm_sum", "read_count"):
        out[f"scan_{k}"] = hits[k]

    # ---- 8. row sets and overlay files (descend_corpus.py:1409-1430,
    #         distill.py:401-457, overlay_sum.py:36-112, descend_corpus.py:627-647)
    import engraft.descend_corpus as dc
    from engraft.replica.overlay_sum import sum_overlays
    frags = FX.fragments(seed=31, n_frag=12, vocab=50, eos=ft7.eos_token_id, lo=3, hi=120)
    all_read = np.asarray(dc.build_all_read_row_set(ft7, frags)["all_read"], dtype=np.int32)
    out["rowset_all_read"] = all_read
    sets = FX.rowset_case_sets(all_read)
    for policy in ("all-read", "private", "entity", "t8-answer"):
        row_map, rows_var = distill.build_rows_var(ft7, frags, policy, sets, FX.ROWSET_EXCLUDE)
        key = policy.replace("-", "_")
        out[f"rowset_{key}_ids"] = np.asarray(list(row_map.keys()), dtype=np.int32)
        out[f"rowset_{key}_rows_sha"] = np.array(sha(rows_var.numpy()))
    true_all = np.stack([ft7.read_rows(*_head_local(ft7, int(g)), 1)[0] for g in all_read]).astype(np.float32)
    with tempfile.TemporaryDirectory() as td:
        paths = []
        for k in range(3):
            rows, data = FX.pleo_fact(k, all_read, true_all)
            pth = Path(td) / f"fact{k}.pleo"
            write_pleo(pth, rows, data)
            paths.append(pth)
        union, merged, manifest = sum_overlays(ft7, paths)
        out["sumov_union"] = union
        out["sumov_merged_sha"] = np.array(sha(merged))
        out["sumov_manifest"] = np.array(repr(manifest))
        row_map, rows_var = distill.build_rows_var(ft7, frags, "private", sets, FX.ROWSET_EXCLUDE)
        rows_var = rows_var + torch.from_numpy(FX.overlay_noise(5, tuple(rows_var.shape)))
        mp = Path(td) / "merged.pleo"
        info = dc.write_merged_pleo(ft7, row_map, rows_var, all_read.tolist(), mp)
        out["merged_bytes_sha"] = np.array(hashlib.sha256(mp.read_bytes()).hexdigest())
        out["merged_n_frozen"] = np.int64(info["n_rows_frozen"])

    # ---- 9. the PLE block that consumes the gathered rows (layers.py:565-626) --------
    import engraft.replica.layers as RL

    class _PleHP:
        hc_mult, n_embd, f_norm_rms_eps, ple_ngram_size = FX.PLE_HC, FX.PLE_N, FX.PLE_EPS, FX.PLE_DIL

    for seed, T, n_hist in FX.PLE_CASES:
        c = FX.ple_case(seed, T, n_hist)
        w = RL.PleWeights(**{k: torch.from_numpy(c[k]) for k in
                             ("w_key", "w_value", "norm_key", "norm_query", "norm_conv", "conv1d")})
        o, h = RL.ple_forward(torch.from_numpy(c["emb"]), torch.from_numpy(c["hidden"]), w,
                              torch.from_numpy(c["hist"]), _PleHP)
        out[f"ple{seed}_out"] = o.numpy()
        out[f"ple{seed}_hist"] = h.numpy()

    meta = dict(reference_root=str(ref_root), torch=torch.__version__, numpy=np.__version__,
                gguf=getattr(gguf, "__version__", "0.19.0"))
    out["meta"] = np.array(repr(meta))
    dst = HERE / "engram_golden.npz"
    np.savez_compressed(dst, **out)
    print(f"wrote {dst} ({dst.stat().st_size} bytes, {len(out)} arrays)")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/make_golden.py <path of the reference checkout>")
    main(sys.argv[1])
