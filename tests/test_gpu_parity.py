"""Parity of the CUDA path (called through the C ABI of libengram_b200.so) with
the CPU oracle and with the reference's golden vectors.

Integer and byte work (row ids, slots, gathered rows, dequantised values,
the bf16 pair-sum epilogue) and the row gradients (summed in the reference's
order) must be bit-identical.  Adam must match the oracle bit for bit and the
reference's torch trajectory within 1e-6 of the row norm (the north-star
tolerance is 1e-5 of the row norm).
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

import fixtures as FX
from cases import fake_table, overlay_case, sha, syn_table
from oracle import oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


@pytest.fixture(scope="module")
def eb():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    import engraft_ngram_b200 as eb
    eb.load_library()
    return eb


def hash_only_table(eb, params, dim=4):
    n_rows = max(o + s for o, s in zip(params["head_offsets"], params["head_sizes"]))
    rows = torch.zeros(n_rows * dim * 4, dtype=torch.uint8, device=DEV)
    return eb.DeviceTable(rows, eb.FMT_F32, dim, params["head_sizes"], params["head_offsets"], params["mult"],
                          params["eos"], params["ngram_size"], params["hpn"], n_rows=n_rows)


def device_table(eb, spec):
    p = spec.params
    return eb.DeviceTable.from_raw(spec.raw, spec.fmt, spec.dim, p["head_sizes"], p["head_offsets"], p["mult"],
                                   p["eos"], p["ngram_size"], p["hpn"], device=DEV)


# ------------------------------------------------------------------ K1: hash
def test_hash_matches_reference_golden(eb, golden):
    t = hash_only_table(eb, FX.fake_table_params(seed=7))
    assert np.array_equal(t.global_ids(golden["hash_fake_tokens"]).cpu().numpy(), golden["hash_fake_ids"])
    t = hash_only_table(eb, FX.syn_params())
    assert np.array_equal(t.global_ids(golden["hash_syn_tokens"]).cpu().numpy(), golden["hash_syn_ids"])
    for k in range(9):
        toks = golden[f"edge{k}_tokens"]
        got = t.global_ids(toks).cpu().numpy() if len(toks) else np.zeros((0, 16), np.int32)
        assert np.array_equal(got, golden[f"edge{k}_ids"].reshape(-1, 16)), k


@pytest.mark.parametrize("seed", [0, 1])
def test_hash_large_random_with_segments_vs_oracle(eb, seed):
    rng = np.random.default_rng(seed)
    sizes = [int(x) for x in rng.integers(2, 40_000_000, size=16)]
    sizes[3] = 1
    sizes[5] = 1 << 20  # a power of two
    params = dict(mult=[int(x) for x in rng.integers(0, 2**64 - 1, size=4, dtype=np.uint64)],
                  head_sizes=sizes, head_offsets=FX.head_offsets(sizes), eos=248044, ngram_size=3, hpn=8)
    T = 131_072
    toks = rng.integers(-5, 2**31 - 1, size=T).astype(np.int32)
    toks[rng.integers(0, T, size=3000)] = 248044
    seg = np.sort(rng.integers(0, 60, size=T))
    ss = FX.seg_starts(seg)
    t = hash_only_table(eb, params, dim=4)
    for t0, n in ((0, T), (777, T - 777 - 5)):
        got = t.global_ids(toks, seg_start=ss, t0=t0, n=n).cpu().numpy()
        ref = O.hash_ids(toks, 3, 8, params["mult"], sizes, params["head_offsets"], 248044, seg_start=ss, t0=t0, n=n)
        assert np.array_equal(got, ref)


# --------------------------------------------- K2 + K3 on the reference's cases
def _golden_case_on_gpu(eb, c):
    dt = device_table(eb, c.table)
    omap = eb.OverlayMap(torch.from_numpy(c.row_ids), DEV)
    rows_var = torch.from_numpy(c.rows_init).to(DEV).requires_grad_(True)
    hits = torch.zeros(1, dtype=torch.int64, device=DEV)
    ss = None if c.seg_start is None else torch.from_numpy(c.seg_start)
    emb = eb.engram_embed(dt, c.tokens, rows_var, omap, ss, c.t0, c.n, hits)
    emb.backward(torch.from_numpy(c.grad).to(DEV))
    return emb.detach().cpu().numpy(), rows_var.grad.cpu().numpy(), int(hits.item())


@pytest.mark.parametrize("prefix", ["ov_syn_", "ov_synnoseg_"])
def test_overlay_emb_iq4nl_matches_reference_bit_exact(eb, golden, prefix):
    c = overlay_case(golden, prefix, syn_table())
    emb, grad_rows, hits = _golden_case_on_gpu(eb, c)
    assert sha(emb) == str(c.golden["emb_sha"])
    assert np.array_equal(emb[1], c.golden["emb_row1"])
    assert hits == int(c.golden["n_id_hits"])
    assert np.array_equal(grad_rows.view(np.uint32), c.golden["grad_rows"].view(np.uint32))


def test_overlay_emb_fake_table_matches_reference_bit_exact(eb, golden, fake1_rows):
    c = overlay_case(golden, "ov_fake_", fake_table(fake1_rows, seed=1))
    emb, grad_rows, hits = _golden_case_on_gpu(eb, c)
    assert sha(emb) == str(c.golden["emb_sha"])
    assert hits == int(c.golden["n_id_hits"])
    assert np.array_equal(grad_rows.view(np.uint32), c.golden["grad_rows"].view(np.uint32))


def test_drop_in_overlay_emb_class(eb, golden):
    """The drop-in class, built exactly as the reference's callers build it
    (engraft/replica/seq.py:1430-1432), reproduces the reference's emb."""
    c = overlay_case(golden, "ov_syn_", syn_table())
    dt = device_table(eb, c.table)
    row_map = {int(g): i for i, g in enumerate(c.row_ids.tolist())}
    rows_var = torch.from_numpy(c.rows_init).to(DEV).requires_grad_(True)
    seg = torch.from_numpy(c.golden["segment_ids"].astype(np.int64))
    ov = eb.OverlayEmb(dt, c.tokens.tolist(), rows_var, row_map, segment_ids=seg, overlay_cache={})
    emb = ov.build(int(c.golden["n_prefix"]))
    assert emb.shape == (c.n, 16 * 160) and emb.dtype == torch.float32 and emb.requires_grad
    assert sha(emb.detach().cpu().numpy()) == str(c.golden["emb_sha"])
    assert ov.n_id_hits == int(c.golden["n_id_hits"]) and ov.n_key_hits == 0
    emb.backward(torch.from_numpy(c.grad).to(DEV))
    assert np.array_equal(rows_var.grad.cpu().numpy().view(np.uint32), c.golden["grad_rows"].view(np.uint32))


def test_device_table_duck_type_matches_table_reads(eb, golden):
    spec = syn_table()
    dt = device_table(eb, spec)
    got = dt.read_rows(3, 0, 64)
    assert np.array_equal(got.view(np.uint32), golden["dq_nl_out"].view(np.uint32))
    toks = golden["hash_syn_tokens"][:50].tolist()
    loc = dt.ngram_addresses(toks)
    ids = golden["hash_syn_ids"][:50] - np.asarray(spec.params["head_offsets"])[None, :]
    assert loc == ids.tolist()


# ------------------------------------------------ random tables vs the oracle
def zipf_tokens(rng, n, vocab=151_936, s=1.1):
    ranks = np.arange(1, vocab + 1, dtype=np.float64)
    cdf = np.cumsum(ranks ** -s)
    cdf /= cdf[-1]
    return np.searchsorted(cdf, rng.random(n)).astype(np.int32)


def random_spec(fmt, dim, n_rows, seed):
    rng = np.random.default_rng(seed)
    if fmt == O.FMT_F32:
        raw = (rng.standard_normal((n_rows, dim)) * 0.0085).astype(np.float32).view(np.uint8).reshape(n_rows, -1)
    elif fmt == O.FMT_IQ4_NL:
        raw = FX.iq4nl_raw(n_rows, seed, dim)
    else:
        raw = FX.iq4xs_raw(n_rows, seed, dim)
    sizes = [n_rows // 16 - 3 * h for h in range(16)]
    sizes[-1] += n_rows - sum(sizes)
    params = dict(mult=[int(x) | 1 for x in rng.integers(1, 2**63, size=4, dtype=np.uint64)], head_sizes=sizes,
                  head_offsets=FX.head_offsets(sizes), eos=151_935, ngram_size=3, hpn=8)
    from cases import TableSpec
    return TableSpec(fmt, dim, raw, params)


FORMATS = [(O.FMT_F32, 128), (O.FMT_F32, 160), (O.FMT_IQ4_NL, 160), (O.FMT_IQ4_XS, 256), (O.FMT_IQ4_XS, 512)]


@pytest.mark.parametrize("fmt,dim", FORMATS)
@pytest.mark.parametrize("mode", [O.MODE_CONCAT_F32, O.MODE_PAIRSUM_ADD_BF16])
def test_forward_backward_random_vs_oracle(eb, fmt, dim, mode):
    seed = 100 * fmt + dim + mode
    rng = np.random.default_rng(seed)
    spec = random_spec(fmt, dim, 40_000, seed)
    T = 3000
    toks = zipf_tokens(rng, T)
    toks[rng.integers(0, T, size=30)] = 151_935
    seg = np.sort(rng.integers(0, 12, size=T))
    ss = FX.seg_starts(seg)
    ids = spec.ids(toks, seg_start=ss)
    read = np.unique(ids)
    ov_ids = np.unique(np.concatenate([rng.choice(read, size=min(len(read), 900), replace=False),
                                       rng.integers(0, 40_000, size=200)])).astype(np.int32)
    rng.shuffle(ov_ids)
    R = len(ov_ids)
    rows_init = (rng.standard_normal((R, dim)) * 0.01).astype(np.float32)

    dt = device_table(eb, spec)
    omap = eb.OverlayMap(torch.from_numpy(ov_ids), DEV)
    rows_var = torch.from_numpy(rows_init).to(DEV).requires_grad_(True)
    hits = torch.zeros(1, dtype=torch.int64, device=DEV)
    if mode == O.MODE_CONCAT_F32:
        out_ref, slots = O.forward(fmt, dim, spec.raw, ids, 8, rows_init, ov_ids, mode)
        out = eb.engram_embed(dt, toks, rows_var, omap, torch.from_numpy(ss), 0, T, hits)
        assert np.array_equal(out.detach().cpu().numpy().view(np.uint32), out_ref.reshape(T, -1).view(np.uint32))
        grad = (rng.standard_normal(out.shape) * 1e-3).astype(np.float32)
        out.backward(torch.from_numpy(grad).to(DEV))
    else:
        res0 = (rng.standard_normal((T, 8 * dim)) * 0.5).astype(np.float32)
        res_bits = O.bf16_bits(res0)
        out_ref, slots = O.forward(fmt, dim, spec.raw, ids, 8, rows_init, ov_ids, mode, residual=res_bits)
        res = torch.from_numpy(res_bits.view(np.int16)).to(DEV).view(torch.bfloat16)
        out = eb.engram_residual_add(res, dt, toks, rows_var, omap, torch.from_numpy(ss), 0, hits)
        assert np.array_equal(out.detach().view(torch.int16).cpu().numpy().view(np.uint16), out_ref)
        grad = O.bf16_bits((rng.standard_normal((T, 8 * dim)) * 1e-2).astype(np.float32))
        out.backward(torch.from_numpy(grad.view(np.int16)).to(DEV).view(torch.bfloat16))
    assert int(hits.item()) == int((slots >= 0).sum())
    gref = O.backward(slots, 8, grad, dim, R, mode)
    assert np.array_equal(rows_var.grad.cpu().numpy().view(np.uint32), gref.view(np.uint32))


def test_backward_heavy_duplicates_and_large_R_bit_exact(eb):
    """A few slots hit thousands of times (sequential order matters) and
    R > 2^16 (three radix passes)."""
    rng = np.random.default_rng(7)
    T, nh, dim = 20_000, 16, 128
    R = 70_000
    slots = np.full((T, nh), -1, dtype=np.int32)
    m = rng.random((T, nh)) < 0.6
    hot = rng.integers(0, 5, size=(T, nh))
    cold = rng.integers(0, R, size=(T, nh))
    slots[m] = np.where(rng.random((T, nh)) < 0.5, hot, cold)[m]
    slots[:, 3] = R - 1
    grad = (rng.standard_normal((T, nh, dim)) * 1e-3).astype(np.float32)
    import engraft_ngram_b200 as ebm
    got = ebm.row_gradients(torch.from_numpy(slots).to(DEV), torch.from_numpy(grad).to(DEV), nh, 8, dim, R,
                            ebm.MODE_CONCAT_F32).cpu().numpy()
    ref = O.backward(slots, 8, grad, dim, R)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    again = ebm.row_gradients(torch.from_numpy(slots).to(DEV), torch.from_numpy(grad).to(DEV), nh, 8, dim, R,
                              ebm.MODE_CONCAT_F32).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), again.view(np.uint32))


@pytest.mark.parametrize("mode,dim", [(0, 4), (0, 36), (0, 128), (0, 200), (0, 256), (0, 512), (0, 1024),
                                      (1, 8), (1, 72), (1, 256), (1, 512), (1, 1024)])
def test_backward_every_row_width_bit_exact(eb, mode, dim):
    """Row widths from one 16-byte vector to 4 KB, with hot slots long enough to
    be split into column slices, against the oracle."""
    rng = np.random.default_rng(1000 + 10 * dim + mode)
    T, nh, hpn = (3000 if dim <= 256 else 900), 16, 8
    R = 5000
    slots = np.full((T, nh), -1, dtype=np.int32)
    m = rng.random((T, nh)) < 0.5
    hot = rng.integers(0, 4, size=(T, nh))
    cold = rng.integers(0, R, size=(T, nh))
    slots[m] = np.where(rng.random((T, nh)) < 0.3, hot, cold)[m]
    slots[rng.random(T) < 0.5, 5] = R - 1
    if mode == O.MODE_CONCAT_F32:
        grad = (rng.standard_normal((T, nh, dim)) * 1e-3).astype(np.float32)
        g_dev = torch.from_numpy(grad).to(DEV)
    else:
        grad = O.bf16_bits((rng.standard_normal((T, hpn * dim)) * 1e-2).astype(np.float32))
        g_dev = torch.from_numpy(grad.view(np.int16)).to(DEV).view(torch.bfloat16)
    got = eb.row_gradients(torch.from_numpy(slots).to(DEV), g_dev, nh, hpn, dim, R, mode).cpu().numpy()
    ref = O.backward(slots, hpn, grad, dim, R, mode)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_backward_no_hits_gives_zero_rows(eb):
    slots = torch.full((100, 16), -1, dtype=torch.int32, device=DEV)
    grad = torch.randn(100, 16, 128, device=DEV)
    g = eb.row_gradients(slots, grad, 16, 8, 128, 33, eb.MODE_CONCAT_F32)
    assert g.shape == (33, 128) and bool((g == 0).all())


# ---------------------------------------------------------------- K4: Adam
def test_adam_matches_oracle_bit_exact_and_reference_within_tolerance(eb, golden):
    rows0 = golden["adam_rows0"]
    p = torch.from_numpy(rows0.copy()).to(DEV).requires_grad_(True)
    opt = eb.OverlayAdam([p], lr=float(golden["adam_lr"]), reg_ref=torch.from_numpy(rows0).to(DEV),
                         reg_mu=float(golden["adam_mu"]))
    po, mo, vo = rows0.copy(), np.zeros_like(rows0), np.zeros_like(rows0)
    rs = np.float32(opt._reg_scale)
    for k in range(golden["adam_grads"].shape[0]):
        p.grad = torch.from_numpy(golden["adam_grads"][k]).to(DEV)
        opt.step()
        O.adam_(po, golden["adam_grads"][k], mo, vo, k + 1, float(golden["adam_lr"]), p0=rows0, reg_scale=rs)
        got = p.detach().cpu().numpy()
        assert np.array_equal(got.view(np.uint32), po.view(np.uint32))
        ref = golden["adam_traj"][k]
        norm = np.linalg.norm(ref, axis=1, keepdims=True)
        assert (np.abs(got - ref) <= 1e-6 * norm).all()


def test_adam_random_sizes_and_misaligned_views(eb):
    rng = np.random.default_rng(3)
    for numel in (1, 7, 4096, 1_000_003):
        p = rng.standard_normal(numel).astype(np.float32) * 0.01
        g = rng.standard_normal(numel).astype(np.float32) * 1e-3
        p0 = rng.standard_normal(numel).astype(np.float32) * 0.01
        m = np.zeros(numel, np.float32)
        v = np.zeros(numel, np.float32)
        big = torch.zeros(numel + 1, device=DEV)
        pd = big[1:]  # 4-byte aligned only: the scalar path
        pd.copy_(torch.from_numpy(p))
        md, vd = torch.zeros(numel, device=DEV), torch.zeros(numel, device=DEV)
        gd, p0d = torch.from_numpy(g).to(DEV), torch.from_numpy(p0).to(DEV)
        lib = eb.load_library()
        for step in (1, 2, 3):
            st = lib.engram_adam_step(pd.data_ptr(), gd.data_ptr(), md.data_ptr(), vd.data_ptr(), p0d.data_ptr(),
                                      numel, step, 1e-3, 0.9, 0.999, 1e-8, 0.37, torch.cuda.current_stream().cuda_stream)
            assert st == 0
            O.adam_(p, g, m, v, step, 1e-3, p0=p0, reg_scale=np.float32(0.37))
        assert np.array_equal(pd.cpu().numpy().view(np.uint32), p.view(np.uint32))
        assert np.array_equal(vd.cpu().numpy().view(np.uint32), v.view(np.uint32))


# ----------------------------------------------------------- pack kernel
@pytest.mark.parametrize("fmt,dim", [(O.FMT_IQ4_NL, 160), (O.FMT_IQ4_NL, 64), (O.FMT_IQ4_XS, 256),
                                     (O.FMT_IQ4_XS, 768), (O.FMT_F32, 12)])
def test_pack_kernel_matches_oracle_layout(eb, fmt, dim):
    spec = random_spec(fmt, dim, 4096, 11)
    dt = device_table(eb, spec)
    got = dt.rows.cpu().numpy().reshape(4096, -1)
    assert np.array_equal(got, O.pack(fmt, dim, spec.raw))


# ---------------------------------------------------- decode-style positions
def test_forward_at_positions_decode_style_vs_oracle(eb):
    """256 sequences x (3 history + 1 new token); rows of the new tokens only."""
    rng = np.random.default_rng(44)
    spec = random_spec(O.FMT_F32, 128, 1 << 16, 44)
    B = 256
    toks = rng.integers(0, 151_935, size=(B, 4)).astype(np.int32)
    toks[::17, 1] = 151_935  # an EOS in some histories
    flat = toks.reshape(-1)
    ss = np.repeat(np.arange(B) * 4, 4).astype(np.int32)
    positions = np.arange(B) * 4 + 3
    ids_all = spec.ids(flat, seg_start=ss)
    ids = ids_all[positions]
    ov_ids = np.unique(ids)[::3].astype(np.int32)
    rows_init = (rng.standard_normal((len(ov_ids), 128)) * 0.01).astype(np.float32)
    out_ref, slots = O.forward(spec.fmt, 128, spec.raw, ids, 8, rows_init, ov_ids)
    dt = device_table(eb, spec)
    omap = eb.OverlayMap(torch.from_numpy(ov_ids), DEV)
    rows_var = torch.from_numpy(rows_init).to(DEV).requires_grad_(True)
    out = eb.engram_embed_at(dt, flat, positions, rows_var, omap, torch.from_numpy(ss))
    assert np.array_equal(out.detach().cpu().numpy().view(np.uint32), out_ref.reshape(B, -1).view(np.uint32))
    grad = (rng.standard_normal(out.shape) * 1e-3).astype(np.float32)
    out.backward(torch.from_numpy(grad).to(DEV))
    gref = O.backward(slots, 8, grad, 128, len(ov_ids))
    assert np.array_equal(rows_var.grad.cpu().numpy().view(np.uint32), gref.view(np.uint32))


# ------------------------------------------------------- row-sharded table
@pytest.mark.parametrize("world", [2, 3, 8])
@pytest.mark.parametrize("fmt,dim,mode", [(O.FMT_IQ4_XS, 256, O.MODE_PAIRSUM_ADD_BF16),
                                          (O.FMT_IQ4_NL, 160, O.MODE_CONCAT_F32),
                                          (O.FMT_F32, 128, O.MODE_CONCAT_F32)])
def test_row_sharded_table_matches_resident_table(eb, world, fmt, dim, mode):
    """W ranks emulated on one GPU: each rank's forward over rows fetched from
    the owners (id mod W) equals the forward over the whole resident table."""
    from engraft_ngram_b200.shard import ShardedTable, local_exchange
    rng = np.random.default_rng(world * 7 + fmt)
    spec = random_spec(fmt, dim, 30_001, 5 + world)
    full = device_table(eb, spec)
    shards = [ShardedTable.from_full(full, world, r) for r in range(world)]
    ex = local_exchange(shards)
    T = 1500
    ov_ids = np.unique(rng.integers(0, 30_001, size=700)).astype(np.int32)
    rows_var = torch.from_numpy((rng.standard_normal((len(ov_ids), dim)) * 0.01).astype(np.float32)).to(DEV)
    omap = eb.OverlayMap(torch.from_numpy(ov_ids), DEV)
    for r in range(world):
        toks = zipf_tokens(rng, T)
        ss = FX.seg_starts(np.sort(rng.integers(0, 5, size=T)))
        ids = spec.ids(toks, seg_start=ss)
        ov_ids_local = ov_ids
        if mode == O.MODE_CONCAT_F32:
            ref, _ = O.forward(fmt, dim, spec.raw, ids, 8, rows_var.cpu().numpy(), ov_ids_local, mode)
            out = torch.empty(T, 16, dim, device=DEV)
        else:
            res = O.bf16_bits((rng.standard_normal((T, 8 * dim)) * 0.5).astype(np.float32))
            ref, _ = O.forward(fmt, dim, spec.raw, ids, 8, rows_var.cpu().numpy(), ov_ids_local, mode, residual=res)
            out = torch.from_numpy(res.view(np.int16)).to(DEV).view(torch.bfloat16)
        shards[r].forward(toks, torch.from_numpy(ss), omap, rows_var, out, mode, ex)
        got = out.view(torch.int32).cpu().numpy() if mode == O.MODE_CONCAT_F32 else out.view(torch.int16).cpu().numpy()
        want = ref.reshape(T, -1).view(np.int32) if mode == O.MODE_CONCAT_F32 else ref.view(np.int16)
        assert np.array_equal(got.reshape(want.shape), want), r


@pytest.mark.parametrize("world", [2, 3, 8])
@pytest.mark.parametrize("fmt,dim", [(O.FMT_IQ4_XS, 256), (O.FMT_IQ4_NL, 160), (O.FMT_F32, 128),
                                     (O.FMT_IQ4_XS, 512), (O.FMT_IQ4_NL, 96)])
@pytest.mark.parametrize("mode", [O.MODE_CONCAT_F32, O.MODE_PAIRSUM_ADD_BF16])
@pytest.mark.parametrize("staged", [False, True])
def test_sharded_table_read_in_place_matches_resident_table(eb, world, fmt, dim, mode, staged):
    """engram_forward_sharded with W ranks' shards emulated as separate buffers
    on one GPU (row g at row g / W of shard g % W): outputs, slots and the hit
    count equal the forward over the whole resident table.  staged: the rows
    of other ranks are first copied by ShardedTable.prefetch on its side
    stream (engram_stage_sharded) and the forward reads them from there
    (engram_forward_staged)."""
    from engraft_ngram_b200.shard import ShardedTable
    rng = np.random.default_rng(31 * world + dim + mode)
    n_rows = 20_003
    spec = random_spec(fmt, dim, n_rows, 9 + world)
    full = device_table(eb, spec)
    shards = [full.rows.view(full.n_rows, full.row_stride)[r::world].contiguous().reshape(-1) for r in range(world)]
    ptrs = torch.tensor([sh.data_ptr() for sh in shards], dtype=torch.int64, device=DEV)
    T = 1100
    toks = zipf_tokens(rng, T)
    ss = torch.from_numpy(FX.seg_starts(np.sort(rng.integers(0, 4, size=T))))
    ov_ids = np.unique(np.concatenate([np.unique(spec.ids(toks))[::4], rng.integers(0, n_rows, size=50)]))
    omap = eb.OverlayMap(torch.from_numpy(ov_ids.astype(np.int32)), DEV)
    rows_var = torch.from_numpy((rng.standard_normal((len(ov_ids), dim)) * 0.01).astype(np.float32)).to(DEV)
    res0 = O.bf16_bits((rng.standard_normal((T, 8 * dim)) * 0.5).astype(np.float32))
    outs = []
    for r in (None, world - 1):
        if mode == O.MODE_CONCAT_F32:
            out = torch.empty(T, 16, dim, device=DEV)
        else:
            out = torch.from_numpy(res0.view(np.int16).copy()).to(DEV).view(torch.bfloat16)
        slots = torch.empty(T, 16, dtype=torch.int32, device=DEV)
        hits = torch.zeros(1, dtype=torch.int64, device=DEV)
        if r is None:
            ov = omap.descriptor(rows_var)
            toks_d, ss_d = torch.from_numpy(toks).to(DEV), ss.to(DEV)  # alive until the kernel has run
            st = eb._lib.load().engram_forward(C.byref(full.ctable), C.byref(ov), toks_d.data_ptr(), ss_d.data_ptr(),
                                               0, T, mode, out.data_ptr(), None, slots.data_ptr(), hits.data_ptr(),
                                               eb._lib.stream_of(DEV))
            eb._lib.check(st, "engram_forward")
        else:
            sh = ShardedTable(shards[r], fmt, dim, full.head_vocab_sizes, full.head_offsets, full.layer_multipliers,
                              full.eos_token_id, world, r, full.n_rows, peer_ptrs=ptrs)
            if staged:
                toks_d, ss_d = torch.from_numpy(toks).to(DEV), ss.to(DEV)
                sh.prefetch(toks_d, ss_d, omap=omap)
                assert len(sh._staged) == 1
                sh.forward(toks_d, ss_d, omap, rows_var, out, mode, slots_out=slots, hit_count=hits)
                assert not sh._staged and len(sh._free) == 1
            else:
                sh.forward(toks, ss, omap, rows_var, out, mode, slots_out=slots, hit_count=hits)
        torch.cuda.synchronize()
        outs.append((out.view(torch.int16).cpu().numpy(), slots.cpu().numpy(), int(hits.item())))
    assert np.array_equal(outs[0][0], outs[1][0])
    assert np.array_equal(outs[0][1], outs[1][1]) and outs[0][2] == outs[1][2]


@pytest.mark.parametrize("world,rank", [(2, 0), (3, 1), (8, 7)])
def test_shard_route_matches_its_contract(eb, world, rank):
    """engram_shard_route over t0 > 0 with segments: one request per (position,
    head) served by another rank and not by the overlay, grouped by owner with
    the restated counts; every request slot is used by exactly one pair and
    send_ids[row_index[k]] is pair k's id."""
    rng = np.random.default_rng(13 * world + rank)
    n_rows = 40_009
    spec = random_spec(O.FMT_IQ4_XS, 256, n_rows, 5 + world)
    full = device_table(eb, spec)
    T, t0 = 2500, 211
    toks = zipf_tokens(rng, T)
    ss = FX.seg_starts(np.sort(rng.integers(0, 6, size=T)))
    ids = spec.ids(toks, seg_start=ss, t0=t0).reshape(-1).astype(np.int64)
    ov_ids = np.unique(np.concatenate([np.unique(ids)[::3], rng.integers(0, n_rows, size=80)])).astype(np.int32)
    omap = eb.OverlayMap(torch.from_numpy(ov_ids), DEV)
    n = T - t0
    entries = n * 16
    words = int(eb._lib.load().engram_shard_route_scratch_words(n, 16, world))
    scratch = torch.empty(words, dtype=torch.int32, device=DEV)
    send = torch.full((entries,), -7, dtype=torch.int32, device=DEV)
    counts = torch.empty(2 * world, dtype=torch.int64, device=DEV)
    rix = torch.empty(entries, dtype=torch.int32, device=DEV)
    ov = eb._lib.EngramOverlay(None, omap.R, omap.keys.data_ptr(), omap.slots.data_ptr(), omap.capacity)
    toks_d, ss_d = torch.from_numpy(toks).to(DEV), torch.from_numpy(ss).to(DEV)
    lib = eb._lib.load()
    assert lib.engram_shard_route(C.byref(full.ctable), C.byref(ov), toks_d.data_ptr(), ss_d.data_ptr(), t0, n, world,
                                  rank, scratch.data_ptr(), words - 1, send.data_ptr(), counts.data_ptr(),
                                  rix.data_ptr(), eb._lib.stream_of(DEV)) == eb._lib.ERR_WORKSPACE
    st = lib.engram_shard_route(C.byref(full.ctable), C.byref(ov), toks_d.data_ptr(), ss_d.data_ptr(), t0, n, world,
                                rank, scratch.data_ptr(), words, send.data_ptr(), counts.data_ptr(), rix.data_ptr(),
                                eb._lib.stream_of(DEV))
    eb._lib.check(st, "engram_shard_route")
    torch.cuda.synchronize()
    req = (ids % world != rank) & ~np.isin(ids, ov_ids)
    want_counts = np.bincount(ids[req] % world, minlength=world)
    got_counts = counts[:world].cpu().numpy()
    assert np.array_equal(got_counts, want_counts)
    got_rix = rix.cpu().numpy()
    assert np.array_equal(got_rix >= 0, req)
    total = int(req.sum())
    assert np.array_equal(np.sort(got_rix[req]), np.arange(total))  # each slot exactly once
    got_send = send[:total].cpu().numpy()
    assert np.array_equal(got_send[got_rix[req]], ids[req])
    off = np.concatenate([[0], np.cumsum(got_counts)])
    for o in range(world):
        assert (got_send[off[o]:off[o + 1]] % world == o).all()


@pytest.mark.parametrize("world,rank", [(2, 1), (3, 2), (8, 5)])
def test_shard_plan_matches_its_contract(eb, world, rank):
    """engram_shard_plan over t0 > 0 with segments: the counts per owner, the
    distinct ids of each owner's group and every pair's row_index equal the
    numpy restatement of the contract (cases.shard_plan_ref); the order inside
    an owner's group is free, so groups compare as sets and row_index through
    send_ids."""
    from cases import shard_plan_ref
    rng = np.random.default_rng(11 * world + rank)
    n_rows = 40_009
    spec = random_spec(O.FMT_IQ4_XS, 256, n_rows, 3 + world)
    full = device_table(eb, spec)
    T, t0 = 2500, 300
    toks = zipf_tokens(rng, T)
    ss = FX.seg_starts(np.sort(rng.integers(0, 6, size=T)))
    ids = spec.ids(toks, seg_start=ss, t0=t0)
    ov_ids = np.unique(np.concatenate([np.unique(ids)[::3], rng.integers(0, n_rows, size=80)])).astype(np.int32)
    omap = eb.OverlayMap(torch.from_numpy(ov_ids), DEV)
    n = T - t0
    entries = n * 16
    cap = 1 << int(np.ceil(np.log2(2 * entries)))
    keys = torch.empty(cap, dtype=torch.int32, device=DEV)
    vals = torch.empty(cap, dtype=torch.int32, device=DEV)
    send = torch.full((entries,), -7, dtype=torch.int32, device=DEV)
    counts = torch.empty(2 * world, dtype=torch.int64, device=DEV)
    rix = torch.empty(entries, dtype=torch.int32, device=DEV)
    ov = eb._lib.EngramOverlay(None, omap.R, omap.keys.data_ptr(), omap.slots.data_ptr(), omap.capacity)
    toks_d, ss_d = torch.from_numpy(toks).to(DEV), torch.from_numpy(ss).to(DEV)
    st = eb._lib.load().engram_shard_plan(C.byref(full.ctable), C.byref(ov), toks_d.data_ptr(), ss_d.data_ptr(), t0,
                                          n, world, rank, keys.data_ptr(), vals.data_ptr(), cap, send.data_ptr(),
                                          counts.data_ptr(), rix.data_ptr(), eb._lib.stream_of(DEV))
    eb._lib.check(st, "engram_shard_plan")
    torch.cuda.synchronize()
    want_send, want_counts, want_rix = shard_plan_ref(ids, ov_ids, world, rank)
    got_counts = counts[:world].cpu().numpy()
    assert np.array_equal(got_counts, want_counts) and got_counts[rank] == 0
    total = int(got_counts.sum())
    got_send = send[:total].cpu().numpy()
    off = np.concatenate([[0], np.cumsum(got_counts)])
    for o in range(world):  # each owner's group holds exactly its ids
        grp = got_send[off[o]:off[o + 1]]
        assert np.array_equal(np.sort(grp), np.sort(want_send[want_send % world == o])), o
    got_rix = rix.cpu().numpy()
    assert np.array_equal(got_rix < 0, want_rix < 0)
    flat = ids.reshape(-1)
    assert np.array_equal(got_send[got_rix[got_rix >= 0]], flat[got_rix >= 0])
    assert total < int((want_rix >= 0).sum())  # a Zipf batch repeats remote rows


@pytest.mark.parametrize("dedup", [False, True])
@pytest.mark.parametrize("world", [2, 3, 8])
@pytest.mark.parametrize("fmt,dim,mode", [(O.FMT_IQ4_XS, 256, O.MODE_PAIRSUM_ADD_BF16),
                                          (O.FMT_IQ4_NL, 160, O.MODE_CONCAT_F32),
                                          (O.FMT_IQ4_XS, 512, O.MODE_PAIRSUM_ADD_BF16)])
def test_exchange_staged_forward_matches_resident_table(eb, world, fmt, dim, mode, dedup):
    """W ranks emulated on one GPU, each with exchange staging over a local
    exchange: four batches pipelined with the prefetch two batches ahead (plan,
    counts, deduplicated exchange, then engram_forward_exchanged) give outputs,
    slots and hit counts bit-identical to the forward over the whole resident
    table; a batch forwarded without a prefetch is planned on the spot."""
    from engraft_ngram_b200.shard import LocalRowExchange, ShardedTable
    rng = np.random.default_rng(41 * world + dim + mode)
    n_rows = 25_013
    spec = random_spec(fmt, dim, n_rows, 13 + world)
    full = device_table(eb, spec)
    shards = [ShardedTable.from_full(full, world, r) for r in range(world)]
    ex = LocalRowExchange(shards)
    T = 1300
    batches = []
    for _ in range(4):
        toks = zipf_tokens(rng, T)
        ss = FX.seg_starts(np.sort(rng.integers(0, 4, size=T)))
        batches.append((torch.from_numpy(toks).to(DEV), torch.from_numpy(ss).to(DEV)))
    read = np.unique(np.concatenate([spec.ids(b[0].cpu().numpy()) for b in batches]))
    ov_ids = np.unique(np.concatenate([read[::5], rng.integers(0, n_rows, size=60)])).astype(np.int32)
    omap = eb.OverlayMap(torch.from_numpy(ov_ids), DEV)
    rows_var = torch.from_numpy((rng.standard_normal((len(ov_ids), dim)) * 0.01).astype(np.float32)).to(DEV)
    res0 = O.bf16_bits((rng.standard_normal((T, 8 * dim)) * 0.5).astype(np.float32))

    def run(forward):
        out = (torch.empty(T, 16, dim, device=DEV) if mode == O.MODE_CONCAT_F32
               else torch.from_numpy(res0.view(np.int16).copy()).to(DEV).view(torch.bfloat16))
        slots = torch.empty(T, 16, dtype=torch.int32, device=DEV)
        hits = torch.zeros(1, dtype=torch.int64, device=DEV)
        forward(out, slots, hits)
        torch.cuda.synchronize()
        return out.view(torch.int16).cpu().numpy(), slots.cpu().numpy(), int(hits.item())

    def resident(b):
        def f(out, slots, hits):
            ov = omap.descriptor(rows_var)
            st = eb._lib.load().engram_forward(C.byref(full.ctable), C.byref(ov), b[0].data_ptr(), b[1].data_ptr(),
                                               0, T, mode, out.data_ptr(), None, slots.data_ptr(), hits.data_ptr(),
                                               eb._lib.stream_of(DEV))
            eb._lib.check(st, "engram_forward")
        return f

    want = [run(resident(b)) for b in batches]
    for r in range(world):
        sh = shards[r]
        sh.enable_exchange_staging(T, ex, dedup=dedup)
        sh.prefetch(*batches[0], omap=omap)
        sh.prefetch(*batches[1], omap=omap)
        for k in range(3):
            if k + 2 < 3:
                sh.prefetch(*batches[k + 2], omap=omap)
            got = run(lambda out, slots, hits: sh.forward(batches[k][0], batches[k][1], omap, rows_var, out, mode,
                                                          slots_out=slots, hit_count=hits))
            assert np.array_equal(got[0], want[k][0]) and np.array_equal(got[1], want[k][1]), (r, k)
            assert got[2] == want[k][2]
        got = run(lambda out, slots, hits: sh.forward(batches[3][0], batches[3][1], omap, rows_var, out, mode,
                                                      slots_out=slots, hit_count=hits))
        assert np.array_equal(got[0], want[3][0]) and got[2] == want[3][2], r


@pytest.mark.parametrize("world", [2, 3, 8])
def test_pushed_route_and_serve_match_their_contract(eb, world):
    """W requesters emulated on one GPU, each with its own batch (t0 > 0,
    segments, an overlay): engram_shard_route_push stores every remote,
    non-overlay (position, head) id in region `requester` of its owner's
    request buffer and the count in the owner's count array, leaves every
    other entry alone, and gives each pair a distinct row in the receive
    layout (owner blocks in ascending order) whose id is the pair's; then
    engram_shard_serve_pushed on every owner writes exactly those rows of the
    resident table into the requester's region of the send buffer."""
    rng = np.random.default_rng(17 * world)
    n_rows = 40_009
    spec = random_spec(O.FMT_IQ4_XS, 256, n_rows, 7 + world)
    full = device_table(eb, spec)
    lib = eb._lib.load()
    T, t0 = 1800, 133
    n = T - t0
    entries = n * 16
    region = entries + 5
    stride = full.row_stride
    req_ids = [torch.full((world * region,), -7, dtype=torch.int32, device=DEV) for _ in range(world)]
    req_cnt = [torch.full((world,), -1, dtype=torch.int64, device=DEV) for _ in range(world)]
    id_ptrs = torch.tensor([x.data_ptr() for x in req_ids], dtype=torch.int64, device=DEV)
    cnt_ptrs = torch.tensor([x.data_ptr() for x in req_cnt], dtype=torch.int64, device=DEV)
    want_ids, got_counts, got_rix = [], [], []
    ov_ids = np.unique(rng.integers(0, n_rows, size=400)).astype(np.int32)
    omap = eb.OverlayMap(torch.from_numpy(ov_ids), DEV)
    ov = eb._lib.EngramOverlay(None, omap.R, omap.keys.data_ptr(), omap.slots.data_ptr(), omap.capacity)
    for r in range(world):
        toks = zipf_tokens(rng, T)
        ss = FX.seg_starts(np.sort(rng.integers(0, 5, size=T)))
        ids = spec.ids(toks, seg_start=ss, t0=t0).reshape(-1).astype(np.int64)
        want_ids.append(ids)
        toks_d, ss_d = torch.from_numpy(toks).to(DEV), torch.from_numpy(ss).to(DEV)
        counts = torch.full((world,), -3, dtype=torch.int64, device=DEV)
        rix = torch.full((entries,), -9, dtype=torch.int32, device=DEV)
        assert lib.engram_shard_route_push(C.byref(full.ctable), C.byref(ov), toks_d.data_ptr(), ss_d.data_ptr(),
                                           t0, n, world, r, id_ptrs.data_ptr(), cnt_ptrs.data_ptr(), entries - 1,
                                           counts.data_ptr(), rix.data_ptr(),
                                           eb._lib.stream_of(DEV)) == eb._lib.ERR_RANGE
        st = lib.engram_shard_route_push(C.byref(full.ctable), C.byref(ov), toks_d.data_ptr(), ss_d.data_ptr(), t0, n,
                                         world, r, id_ptrs.data_ptr(), cnt_ptrs.data_ptr(), region, counts.data_ptr(),
                                         rix.data_ptr(), eb._lib.stream_of(DEV))
        eb._lib.check(st, "engram_shard_route_push")
        got_counts.append(counts)
        got_rix.append(rix)
    torch.cuda.synchronize()
    ids_h = [x.cpu().numpy().reshape(world, region) for x in req_ids]
    cnt_h = [x.cpu().numpy() for x in req_cnt]
    for r in range(world):
        ids = want_ids[r]
        req = (ids % world != r) & ~np.isin(ids, ov_ids)
        want_counts = np.bincount(ids[req] % world, minlength=world)
        counts = got_counts[r].cpu().numpy()
        assert np.array_equal(counts, want_counts) and counts[r] == 0
        base = np.concatenate([[0], np.cumsum(counts)])
        rix = got_rix[r].cpu().numpy()
        assert np.array_equal(rix >= 0, req)
        assert np.array_equal(np.sort(rix[req]), np.arange(int(req.sum())))  # each receive row exactly once
        owner = ids % world
        for o in range(world):
            if o == r:
                assert (ids_h[o][r] == -7).all() and cnt_h[o][r] == -1  # nothing stored for itself
                continue
            c = int(counts[o])
            assert cnt_h[o][r] == c
            blk = ids_h[o][r]
            assert (blk[c:] == -7).all()
            sel = req & (owner == o)
            assert np.array_equal(blk[rix[sel] - base[o]], ids[sel])  # the pair's row holds its id
    # every owner serves its requesters' regions from its shard
    rows = full.rows.cpu().numpy().reshape(full.n_rows, stride)
    for o in range(world):
        shard = full.rows.view(full.n_rows, stride)[o::world].contiguous()
        send = torch.full((world * region * stride,), 0xCD, dtype=torch.uint8, device=DEV)
        st = lib.engram_shard_serve_pushed(shard.data_ptr(), stride, shard.shape[0], world, o, req_ids[o].data_ptr(),
                                           req_cnt[o].data_ptr(), region, send.data_ptr(), eb._lib.stream_of(DEV))
        eb._lib.check(st, "engram_shard_serve_pushed")
        torch.cuda.synchronize()
        got = send.cpu().numpy().reshape(world, region, stride)
        for r in range(world):
            c = 0 if r == o else int(cnt_h[o][r])
            assert np.array_equal(got[r, :c], rows[ids_h[o][r][:c].astype(np.int64)]), (o, r)
            assert (got[r, c:] == 0xCD).all()


@pytest.mark.parametrize("world", [2, 3, 8])
@pytest.mark.parametrize("fmt,dim,mode", [(O.FMT_IQ4_XS, 256, O.MODE_PAIRSUM_ADD_BF16),
                                          (O.FMT_IQ4_NL, 160, O.MODE_CONCAT_F32)])
def test_pushed_exchange_staged_forward_matches_resident_table(eb, world, fmt, dim, mode):
    """W ranks emulated on one GPU with the pushing exchange
    (LocalPeerRowExchange), their calls interleaved as real ranks' are: six
    batches per rank prefetched three ahead, the first five forwarded (the
    fifth still waiting for its fetch, done on the spot); every forward's
    output, slots and hit count are bit-identical to the forward over the whole
    resident table.  (A batch forwarded before its owners served it needs the
    other ranks inside the same call: the two-rank test covers it.)"""
    from engraft_ngram_b200.shard import LocalPeerRowExchange, ShardedTable
    rng = np.random.default_rng(43 * world + dim)
    n_rows = 25_013
    spec = random_spec(fmt, dim, n_rows, 17 + world)
    full = device_table(eb, spec)
    shards = [ShardedTable.from_full(full, world, r) for r in range(world)]
    T, K, depth = 900, 6, 3
    exs = LocalPeerRowExchange.for_shards(shards, T)
    for sh, ex in zip(shards, exs):
        sh.enable_exchange_staging(T, ex)
    batches = []
    for r in range(world):
        bs = []
        for _ in range(K):
            toks = zipf_tokens(rng, T)
            ss = FX.seg_starts(np.sort(rng.integers(0, 4, size=T)))
            bs.append((torch.from_numpy(toks).to(DEV), torch.from_numpy(ss).to(DEV)))
        batches.append(bs)
    read = np.unique(np.concatenate([spec.ids(b[0].cpu().numpy()).reshape(-1) for bs in batches for b in bs]))
    ov_ids = np.unique(np.concatenate([read[::5], rng.integers(0, n_rows, size=60)])).astype(np.int32)
    omap = eb.OverlayMap(torch.from_numpy(ov_ids), DEV)
    rows_var = torch.from_numpy((rng.standard_normal((len(ov_ids), dim)) * 0.01).astype(np.float32)).to(DEV)
    res0 = O.bf16_bits((rng.standard_normal((T, 8 * dim)) * 0.5).astype(np.float32))

    def fresh():
        if mode == O.MODE_CONCAT_F32:
            return torch.empty(T, 16, dim, device=DEV)
        return torch.from_numpy(res0.view(np.int16).copy()).to(DEV).view(torch.bfloat16)

    def resident(b):
        out, slots = fresh(), torch.empty(T, 16, dtype=torch.int32, device=DEV)
        hits = torch.zeros(1, dtype=torch.int64, device=DEV)
        ov = omap.descriptor(rows_var)
        st = eb._lib.load().engram_forward(C.byref(full.ctable), C.byref(ov), b[0].data_ptr(), b[1].data_ptr(), 0, T,
                                           mode, out.data_ptr(), None, slots.data_ptr(), hits.data_ptr(),
                                           eb._lib.stream_of(DEV))
        eb._lib.check(st, "engram_forward")
        return out, slots, hits

    want = [[resident(b) for b in bs] for bs in batches]
    got = [[None] * K for _ in range(world)]
    for k in range(depth):
        for r in range(world):
            shards[r].prefetch(*batches[r][k], omap=omap)
    for k in range(K - 1):
        for r in range(world):  # every rank's prefetch of this step, then every rank's forward
            if k + depth < K:
                shards[r].prefetch(*batches[r][k + depth], omap=omap)
        for r in range(world):
            out, slots = fresh(), torch.empty(T, 16, dtype=torch.int32, device=DEV)
            hits = torch.zeros(1, dtype=torch.int64, device=DEV)
            shards[r].forward(batches[r][k][0], batches[r][k][1], omap, rows_var, out, mode, slots_out=slots,
                              hit_count=hits)
            got[r][k] = (out, slots, hits)
    torch.cuda.synchronize()
    for r in range(world):
        for k in range(K - 1):
            g, w = got[r][k], want[r][k]
            assert torch.equal(g[0].view(torch.int16), w[0].view(torch.int16)), (r, k)
            assert torch.equal(g[1], w[1]) and int(g[2].item()) == int(w[2].item()), (r, k)


@pytest.mark.parametrize("world,rank", [(2, 1), (3, 0), (8, 5)])
def test_stage_copies_exactly_the_rows_of_other_ranks(eb, world, rank):
    """engram_stage_sharded over t0 > 0: head h of output row i holds the
    resident bytes of its global row when another rank owns it and the overlay
    does not serve it; the bytes of every other head are left as they were."""
    rng = np.random.default_rng(5 * world + rank)
    spec = random_spec(O.FMT_IQ4_XS, 256, 12_007, 40 + world)
    full = device_table(eb, spec)
    shards = [full.rows.view(full.n_rows, full.row_stride)[r::world].contiguous().reshape(-1) for r in range(world)]
    ptrs = torch.tensor([sh.data_ptr() for sh in shards], dtype=torch.int64, device=DEV)
    T, t0 = 700, 37
    toks = zipf_tokens(rng, T)
    ss_np = FX.seg_starts(np.sort(rng.integers(0, 3, size=T)))
    toks_d, ss_d = torch.from_numpy(toks).to(DEV), torch.from_numpy(ss_np).to(DEV)
    n = T - t0
    lib = eb._lib.load()
    nbytes = int(lib.engram_stage_bytes(C.byref(full.ctable), n))
    assert nbytes == n * 16 * full.row_stride
    stage = torch.full((nbytes,), 0xAB, dtype=torch.uint8, device=DEV)
    ids = spec.ids(toks, ss_np)[t0:]
    ov_ids = np.unique(ids.reshape(-1))[::5].astype(np.int32)
    omap = eb.OverlayMap(torch.from_numpy(ov_ids), DEV)
    ov = omap.descriptor(torch.zeros(len(ov_ids), 256, device=DEV))
    st = lib.engram_stage_sharded(C.byref(full.ctable), C.byref(ov), toks_d.data_ptr(), ss_d.data_ptr(), t0, n,
                                  ptrs.data_ptr(), world, rank, stage.data_ptr(), 7, eb._lib.stream_of(DEV))
    eb._lib.check(st, "engram_stage_sharded")
    torch.cuda.synchronize()
    got = stage.cpu().numpy().reshape(n, 16, full.row_stride)
    rows = full.rows.cpu().numpy().reshape(full.n_rows, full.row_stride)
    remote = (ids % world != rank) & ~np.isin(ids, ov_ids)
    assert remote.any() and (~remote).any() and np.isin(ids, ov_ids).any()
    assert np.array_equal(got[remote], rows[ids[remote]])
    assert (got[~remote] == 0xAB).all()


@pytest.mark.parametrize("world", [2, 3, 8, 16])
@pytest.mark.parametrize("fmt,dim", [(O.FMT_IQ4_XS, 256), (O.FMT_IQ4_NL, 96)])
def test_push_stage_plan_and_copy(eb, world, fmt, dim):
    """W emulated ranks on one GPU, each with its own batch: engram_stage_plan
    lays out each requester's stage by owner (block o = rank o's rows in
    output-row-then-head order), every owner's engram_stage_push fills its
    block of every stage, and the forward over the stage through the row index
    (engram_forward_indirect) equals the resident-table forward."""
    from engraft_ngram_b200.shard import ShardedTable
    rng = np.random.default_rng(17 * world + dim)
    n_rows = 24_001
    spec = random_spec(fmt, dim, n_rows, 70 + world)
    full = device_table(eb, spec)
    stride = full.row_stride
    shards = [full.rows.view(n_rows, stride)[r::world].contiguous().reshape(-1) for r in range(world)]
    sptrs = torch.tensor([sh.data_ptr() for sh in shards], dtype=torch.int64, device=DEV)
    T, t0 = 900, 5
    n = T - t0
    toks = [zipf_tokens(rng, T) for _ in range(world)]
    seg = [FX.seg_starts(np.sort(rng.integers(0, 3, size=T))) for _ in range(world)]
    tok_d = [torch.from_numpy(x).to(DEV) for x in toks]
    seg_d = [torch.from_numpy(x).to(DEV) for x in seg]
    lib = eb._lib.load()
    words = int(lib.engram_stage_plan_words(n, world))
    assert words == world * ((n + 31) // 32 + 1)
    plans = [torch.full((words,), -7, dtype=torch.int32, device=DEV) for _ in range(world)]
    rix = [torch.full((n * 16,), -7, dtype=torch.int32, device=DEV) for _ in range(world)]
    stages = [torch.full((n * 16 * stride,), 0xCD, dtype=torch.uint8, device=DEV) for _ in range(world)]
    ptr = lambda xs: torch.tensor([x.data_ptr() for x in xs], dtype=torch.int64, device=DEV)
    tp, gp, pp, stp = ptr(tok_d), ptr(seg_d), ptr(plans), ptr(stages)
    tables = [ShardedTable(shards[r], fmt, dim, full.head_vocab_sizes, full.head_offsets, full.layer_multipliers,
                           full.eos_token_id, world, r, n_rows, peer_ptrs=sptrs) for r in range(world)]
    for r in range(world):
        st = lib.engram_stage_plan(C.byref(tables[r].ctable), tok_d[r].data_ptr(), seg_d[r].data_ptr(), t0, n, world,
                                   plans[r].data_ptr(), rix[r].data_ptr(), eb._lib.stream_of(DEV))
        eb._lib.check(st, "engram_stage_plan")
    for o in range(world):  # every owner pushes its rows into every rank's stage, its own included
        st = lib.engram_stage_push(C.byref(tables[o].ctable), tp.data_ptr(), gp.data_ptr(), pp.data_ptr(), t0, n,
                                   stp.data_ptr(), world, o, 3 if o % 2 else 0, eb._lib.stream_of(DEV))
        eb._lib.check(st, "engram_stage_push")
    torch.cuda.synchronize()
    rows = full.rows.cpu().numpy().reshape(n_rows, stride)
    ov_ids = np.unique(rng.integers(0, n_rows, size=400)).astype(np.int32)
    omap = eb.OverlayMap(torch.from_numpy(ov_ids), DEV)
    rows_var = torch.from_numpy((rng.standard_normal((len(ov_ids), dim)) * 0.01).astype(np.float32)).to(DEV)
    tiles = (n + 31) // 32
    for r in range(world):
        ids = spec.ids(toks[r], seg_start=seg[r])[t0:].astype(np.int64)
        owner = ids % world
        # the plan: blocks by owner, each in (output row, head) order
        order = np.lexsort((np.arange(n * 16), owner.reshape(-1)))
        want_rix = np.empty(n * 16, dtype=np.int64)
        want_rix[order] = np.arange(n * 16)
        got_rix = rix[r].cpu().numpy()
        assert np.array_equal(got_rix, want_rix)
        plan = plans[r].cpu().numpy().reshape(world, tiles + 1)
        counts = np.bincount(owner.reshape(-1), minlength=world)
        assert np.array_equal(plan[:, tiles], np.cumsum(counts))
        assert np.array_equal(plan[:, 0], np.cumsum(counts) - counts)
        stage = stages[r].cpu().numpy().reshape(n * 16, stride)
        assert np.array_equal(stage[got_rix], rows[ids.reshape(-1)])
        want = torch.empty(n, 16, dim, device=DEV)
        ov = omap.descriptor(rows_var)
        st = lib.engram_forward(C.byref(full.ctable), C.byref(ov), tok_d[r].data_ptr(), seg_d[r].data_ptr(), t0, n,
                                O.MODE_CONCAT_F32, want.data_ptr(), None, None, None, eb._lib.stream_of(DEV))
        eb._lib.check(st, "engram_forward")
        desc = eb._lib.EngramTable.from_buffer_copy(tables[r].ctable)
        desc.rows = stages[r].data_ptr()
        desc.n_rows = n * 16
        out = torch.empty(n, 16, dim, device=DEV)
        st = lib.engram_forward_indirect(C.byref(desc), C.byref(ov), tok_d[r].data_ptr(), seg_d[r].data_ptr(), t0, n,
                                         rix[r].data_ptr(), O.MODE_CONCAT_F32, out.data_ptr(), None, None, None,
                                         eb._lib.stream_of(DEV))
        eb._lib.check(st, "engram_forward_indirect")
        torch.cuda.synchronize()
        assert torch.equal(out.view(torch.int32), want.view(torch.int32)), r


def test_sharded_table_through_the_public_autograd_api(eb):
    """engram_residual_add and engram_embed given a ShardedTable (W = 2
    emulated): outputs and row gradients equal the resident table's."""
    from engraft_ngram_b200.shard import ShardedTable, local_exchange
    rng = np.random.default_rng(77)
    spec = random_spec(O.FMT_IQ4_XS, 256, 30_001, 77)
    full = device_table(eb, spec)
    shards = [ShardedTable.from_full(full, 2, r) for r in range(2)]
    ex = local_exchange(shards)
    for sh in shards:
        sh.exchange = ex
    T = 1200
    toks = zipf_tokens(rng, T)
    ss = torch.from_numpy(FX.seg_starts(np.sort(rng.integers(0, 4, size=T))))
    ov_ids = np.unique(np.concatenate([np.unique(spec.ids(toks))[::3], rng.integers(0, 30_001, size=100)]))
    omap = eb.OverlayMap(torch.from_numpy(ov_ids.astype(np.int32)), DEV)
    rows0 = (rng.standard_normal((len(ov_ids), 256)) * 0.01).astype(np.float32)
    res0 = O.bf16_bits((rng.standard_normal((T, 8 * 256)) * 0.5).astype(np.float32))
    gout = O.bf16_bits((rng.standard_normal((T, 8 * 256)) * 1e-2).astype(np.float32))
    results = []
    for table in (full, shards[1]):
        rv = torch.from_numpy(rows0).to(DEV).requires_grad_(True)
        res = torch.from_numpy(res0.view(np.int16)).to(DEV).view(torch.bfloat16)
        out = eb.engram_residual_add(res, table, toks, rv, omap, ss)
        out.backward(torch.from_numpy(gout.view(np.int16)).to(DEV).view(torch.bfloat16))
        rv2 = torch.from_numpy(rows0).to(DEV).requires_grad_(True)
        emb = eb.engram_embed(table, toks, rv2, omap, ss)
        results.append((out.detach().view(torch.int16).cpu().numpy(), rv.grad.cpu().numpy(),
                        emb.detach().cpu().numpy()))
    (o_a, g_a, e_a), (o_b, g_b, e_b) = results
    assert np.array_equal(o_a, o_b)
    assert np.array_equal(g_a.view(np.uint32), g_b.view(np.uint32))
    assert np.array_equal(e_a.view(np.uint32), e_b.view(np.uint32))


# ------------------------------------------------- bulk hash + overlay hit scan
def test_scan_hits_matches_reference_golden(eb, golden):
    p = FX.fake_table_params(seed=7)
    t = hash_only_table(eb, p)
    for block in (20_000, 4_000, 777):
        got = eb.scan_hits(golden["scan_tokens"], t, golden["scan_overlay"], golden["scan_dnorm"], block=block)
        assert np.array_equal(got["pos"], golden["scan_pos"]), block
        assert np.array_equal(got["n_hit_rows"], golden["scan_n_hit_rows"])
        assert np.array_equal(got["dnorm_max"].view(np.uint32), golden["scan_dnorm_max"].view(np.uint32))
        assert np.array_equal(got["dnorm_sum"].view(np.uint32), golden["scan_dnorm_sum"].view(np.uint32))
        assert np.array_equal(got["read_count"], golden["scan_read_count"])


class _AddressingOnly:
    """The attributes of a reference table that hashing reads (a PleTable or
    FakeTable without rows)."""

    def __init__(self, p):
        self.head_vocab_sizes = list(p["head_sizes"])
        self.head_offsets = list(p["head_offsets"])
        self.layer_multipliers = list(p["mult"])
        self.eos_token_id = p["eos"]
        self.ngram_size = p["ngram_size"]
        self.heads_per_ngram = p["hpn"]


def test_scan_hits_installed_takes_the_reference_table_object(eb, golden):
    """install_scan reroutes engraft.damage.scan_hits; the reference passes its
    own table object, of which only the addressing constants are used."""
    import types
    dmg = types.SimpleNamespace(scan_hits=None)
    eb.install_scan(dmg)
    try:
        table = _AddressingOnly(FX.fake_table_params(seed=7))
        got = dmg.scan_hits(golden["scan_tokens"], table, golden["scan_overlay"], golden["scan_dnorm"])
    finally:
        eb.uninstall_scan(dmg)
    assert np.array_equal(got["pos"], golden["scan_pos"])
    assert np.array_equal(got["n_hit_rows"], golden["scan_n_hit_rows"])
    assert np.array_equal(got["dnorm_sum"].view(np.uint32), golden["scan_dnorm_sum"].view(np.uint32))
    assert np.array_equal(got["read_count"], golden["scan_read_count"])


def test_scan_hits_large_corpus_vs_oracle(eb):
    rng = np.random.default_rng(9)
    p = FX.syn_params()
    t = hash_only_table(eb, p)
    toks = zipf_tokens(rng, 2_000_000)
    toks[rng.integers(0, toks.size, size=5000)] = p["eos"]
    ids = O.hash_ids(toks[:200_000], 3, 8, p["mult"], p["head_sizes"], p["head_offsets"], p["eos"])
    ov = np.unique(np.concatenate([np.unique(ids)[::50], rng.integers(0, sum(FX.SYN_HEAD_SIZES), size=300)]))
    dn = (rng.random(len(ov)) * 0.2).astype(np.float32)
    got = eb.scan_hits(toks, t, ov, dn, block=300_000)
    ref = O.scan_hits(toks, 3, 8, p["mult"], p["head_sizes"], p["head_offsets"], p["eos"], ov, dn)
    for k in ("pos", "n_hit_rows", "read_count"):
        assert np.array_equal(got[k], ref[k]), k
    for k in ("dnorm_max", "dnorm_sum"):
        assert np.array_equal(got[k].view(np.uint32), ref[k].view(np.uint32)), k


# ------------------------------------------------- row sets and overlay files
class _FakeTable7:
    """FakeTable(seed=7)'s interface (engraft/testing/fake_table.py): addressing
    constants plus read_rows, over its rows restated by the fixtures."""

    def __init__(self):
        p = FX.fake_table_params(seed=7)
        self.rows = FX.fake_table_rows(seed=7)
        self.head_vocab_sizes = list(p["head_sizes"])
        self.head_offsets = list(p["head_offsets"])
        self.layer_multipliers = list(p["mult"])
        self.eos_token_id = p["eos"]
        self.ngram_size = p["ngram_size"]
        self.heads_per_ngram = p["hpn"]

    def read_rows(self, h, start, n):
        o = self.head_offsets[h] + start
        return self.rows[o:o + n]


@pytest.fixture(scope="module")
def fake7():
    return _FakeTable7()


def _frags7():
    return FX.fragments(seed=31, n_frag=12, vocab=50, eos=FX.fake_table_params(seed=7)["eos"], lo=3, hi=120)


def test_build_all_read_row_set_matches_reference_golden(eb, golden, fake7):
    from engraft_ngram_b200 import rowset
    got = rowset.build_all_read_row_set(fake7, _frags7())
    assert got["all_read"] == golden["rowset_all_read"].tolist()


@pytest.mark.parametrize("policy", ["all-read", "private", "entity", "t8-answer"])
def test_build_rows_var_matches_reference_golden(eb, golden, fake7, policy):
    import hashlib
    from engraft_ngram_b200 import rowset
    sets = FX.rowset_case_sets(golden["rowset_all_read"])
    row_map, rows_var = rowset.build_rows_var(fake7, _frags7(), policy, sets, FX.ROWSET_EXCLUDE)
    key = policy.replace("-", "_")
    assert list(row_map.keys()) == golden[f"rowset_{key}_ids"].tolist()
    assert list(row_map.values()) == list(range(len(row_map)))
    assert rows_var.device.type == "cpu" and rows_var.dtype == torch.float32
    assert hashlib.sha256(rows_var.numpy().tobytes()).hexdigest() == str(golden[f"rowset_{key}_rows_sha"])


def test_sum_overlays_matches_reference_golden(eb, golden, fake7, tmp_path):
    import ast
    import hashlib
    from engraft_ngram_b200 import rowset
    all_read = golden["rowset_all_read"]
    paths = []
    for k in range(3):
        rows, data = FX.pleo_fact(k, all_read, fake7.rows[all_read])
        pth = tmp_path / f"fact{k}.pleo"
        eb.write_pleo(pth, rows, data)
        paths.append(pth)
    union, merged, manifest = rowset.sum_overlays(fake7, paths)
    assert np.array_equal(union, golden["sumov_union"]) and union.dtype == np.int32
    assert hashlib.sha256(merged.tobytes()).hexdigest() == str(golden["sumov_merged_sha"])
    ref = ast.literal_eval(str(golden["sumov_manifest"]))
    for k in ("n_files", "n_rows_union", "n_rows_moved_any", "n_rows_shared", "facts_per_row_histogram",
              "quant_floor", "max_row_delta_norm_over_quant_floor"):
        assert manifest[k] == ref[k], k
    for k in ("shared_rows_sum_abs_norm_mean", "shared_rows_sum_abs_norm_max", "shared_rows_abs_sum_norm_mean",
              "shared_rows_abs_sum_norm_max", "max_row_delta_norm"):
        assert manifest[k] == pytest.approx(ref[k], rel=1e-12, abs=1e-15), k  # float64 norms, summed in another order


def test_overlay_accumulate_adds_repeated_rows_in_file_order(eb):
    """engram_overlay_accumulate with the stable device sort of the targets
    (rowset._accumulate): a file whose rows repeat (up to 40 times, index -1
    skipped) gives bit for bit numpy's np.add.at of the fp32 deltas, which
    adds repeated rows in file order."""
    from engraft_ngram_b200 import rowset
    rng = np.random.default_rng(71)
    n, R, dim = 6000, 300, 160
    idx = rng.zipf(1.3, size=n).astype(np.int64) % R
    idx[rng.random(n) < 0.05] = -1
    data = (rng.standard_normal((n, dim)) * 1e-2).astype(np.float32)
    base = (rng.standard_normal((n, dim)) * 1e-2).astype(np.float32)
    acc0 = (rng.standard_normal((R, dim)) * 1e-3).astype(np.float32)
    want = acc0.copy()
    keep = idx >= 0
    np.add.at(want, idx[keep], data[keep] - base[keep])
    acc = torch.from_numpy(acc0.copy()).to(DEV)
    rowset._accumulate(acc, torch.from_numpy(idx.astype(np.int32)).to(DEV), torch.from_numpy(data).to(DEV),
                       torch.from_numpy(base).to(DEV))
    torch.cuda.synchronize()
    assert np.bincount(idx[keep]).max() >= 20
    assert np.array_equal(acc.cpu().numpy().view(np.uint32), want.view(np.uint32))


def test_write_merged_pleo_matches_reference_golden(eb, golden, fake7, tmp_path):
    import hashlib
    from engraft_ngram_b200 import rowset
    sets = FX.rowset_case_sets(golden["rowset_all_read"])
    row_map, rows_var = rowset.build_rows_var(fake7, _frags7(), "private", sets, FX.ROWSET_EXCLUDE)
    rows_var = rows_var + torch.from_numpy(FX.overlay_noise(5, tuple(rows_var.shape)))
    out = tmp_path / "merged.pleo"
    info = rowset.write_merged_pleo(fake7, row_map, rows_var, golden["rowset_all_read"].tolist(), out)
    assert info["n_rows_frozen"] == int(golden["merged_n_frozen"])
    assert hashlib.sha256(out.read_bytes()).hexdigest() == str(golden["merged_bytes_sha"])


def test_device_row_set_algebra_and_index_vs_numpy(eb):
    """Unions, differences, intersections, the sorted list and member indices
    on a 320 M-row table (40 MB bitmaps), against numpy set operations."""
    from engraft_ngram_b200.rowset import DeviceRowSet
    rng = np.random.default_rng(3)
    n_rows = 320_001_536
    a_ids = np.unique(rng.integers(0, n_rows, size=200_000))
    b_ids = np.unique(np.concatenate([a_ids[::3], rng.integers(0, n_rows, size=50_000), [0, n_rows - 1]]))
    a = DeviceRowSet.of_ids(a_ids, n_rows, DEV)
    b = DeviceRowSet.of_ids(b_ids, n_rows, DEV)
    assert np.array_equal(a.ids().cpu().numpy(), a_ids)
    assert np.array_equal((a | b).ids().cpu().numpy(), np.union1d(a_ids, b_ids))
    assert np.array_equal((a - b).ids().cpu().numpy(), np.setdiff1d(a_ids, b_ids))
    assert np.array_equal((a & b).ids().cpu().numpy(), np.intersect1d(a_ids, b_ids))
    assert len(b) == b_ids.size
    probe = np.concatenate([b_ids[::7], rng.integers(0, n_rows, size=1000)]).astype(np.int32)
    idx = b.index(torch.from_numpy(probe)).cpu().numpy()
    pos = np.searchsorted(b_ids, probe)
    member = (pos < b_ids.size) & (b_ids[np.minimum(pos, b_ids.size - 1)] == probe)
    assert np.array_equal(idx, np.where(member, pos, -1))


def test_owner_exchange_emulated_ranks_match_summed_dense_adam(eb):
    """The peer-memory update with W = 3 ranks emulated on one GPU (separate
    buffers, one launch per rank): every rank's backward stores its row
    gradients into the owners' receive buffers; each owner's step sums them in
    rank order and runs Adam.  Every rank's rows equal Adam over the rank-order
    sum of the dense row gradients, bit for bit; so do m and v."""
    from engraft_ngram_b200 import _lib as L
    from engraft_ngram_b200.dist import adam_owner_step, backward_to_owners, shard_bounds
    rng = np.random.default_rng(12)
    W, R, dim, T, nh, hpn = 3, 1001, 256, 700, 16, 8
    mode = L.MODE_PAIRSUM_ADD_BF16
    p_init = (rng.standard_normal((R, dim)) * 0.01).astype(np.float32)
    p0 = torch.from_numpy(p_init.copy()).to(DEV)
    size_max = -(-R // W)
    recv = [torch.full((W * size_max, dim), float("nan"), device=DEV) for _ in range(W)]
    rows = [torch.from_numpy(p_init.copy()).to(DEV) for _ in range(W)]
    recv_p = torch.tensor([t.data_ptr() for t in recv], dtype=torch.int64, device=DEV)
    rows_p = torch.tensor([t.data_ptr() for t in rows], dtype=torch.int64, device=DEV)
    spans = [shard_bounds(R, W, r) for r in range(W)]
    ms = [torch.zeros(hi - lo, dim, device=DEV) for lo, hi in spans]
    vs = [torch.zeros_like(m) for m in ms]
    ref_p = p0.clone()
    ref_m, ref_v = torch.zeros_like(ref_p), torch.zeros_like(ref_p)
    rs = float(eb.reg_scale(0.1, p0))
    for step in (1, 2):
        dense = []
        for r in range(W):
            slots = np.full((T, nh), -1, dtype=np.int32)
            hit = rng.random((T, nh)) < 0.4
            slots[hit] = rng.integers(0, R - 7, size=int(hit.sum()))  # the last rows stay without entries
            slots[:, 2] = rng.integers(0, 3, size=T)  # hot rows: long segments
            sl = torch.from_numpy(slots).to(DEV)
            g = torch.from_numpy(O.bf16_bits((rng.standard_normal((T, hpn * dim)) * 1e-2).astype(np.float32))
                                 .view(np.int16)).to(DEV).view(torch.bfloat16)
            backward_to_owners(sl, g, nh, hpn, dim, R, mode, recv_p, W, r)
            dense.append(eb.row_gradients(sl, g, nh, hpn, dim, R, mode))
        for o, (lo, hi) in enumerate(spans):  # block k of owner o = rank k's rows [lo, hi)
            for k in range(W):
                blk = recv[o][k * (hi - lo):(k + 1) * (hi - lo)]
                assert torch.equal(blk.view(torch.int32), dense[k][lo:hi].view(torch.int32)), (step, o, k)
        for o, (lo, hi) in enumerate(spans):
            adam_owner_step(recv[o], rows_p, W, o, R, dim, ms[o], vs[o], p0[lo:hi], step, 1e-3, reg_scale=rs)
        gsum = dense[0].clone()
        for k in range(1, W):
            gsum = gsum + dense[k]
        st = L.load().engram_adam_step(ref_p.data_ptr(), gsum.data_ptr(), ref_m.data_ptr(), ref_v.data_ptr(),
                                       p0.data_ptr(), ref_p.numel(), step, 1e-3, 0.9, 0.999, 1e-8, rs,
                                       L.stream_of(ref_p.device))
        L.check(st, "engram_adam_step")
        for r in range(W):
            assert torch.equal(rows[r].view(torch.int32), ref_p.view(torch.int32)), (step, r)
        for o, (lo, hi) in enumerate(spans):
            assert torch.equal(ms[o].view(torch.int32), ref_m[lo:hi].view(torch.int32))
            assert torch.equal(vs[o].view(torch.int32), ref_v[lo:hi].view(torch.int32))
