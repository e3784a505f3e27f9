"""Deterministic inputs shared by the golden-vector generator (make_golden.py)
and the tests.  Test infrastructure: nothing in the product imports this.

Two table families, both seeded, so a test can rebuild byte-identical inputs
from the few parameters stored in a fixture:

* the reference's FakeTable (engraft/testing/fake_table.py:23-76): 16 heads of
  5,000 fp32 rows of width 160, rows drawn per (seed, head, row);
* a synthetic per-head IQ4_NL table of the real format (engraft/table.py:40-88):
  16 prime, non-power-of-two head sizes, multipliers with bit 63 set, the real
  corpus EOS id, random nibbles and finite fp16 block scales.
"""
from __future__ import annotations

import numpy as np

ROW_LEN = 160
N_HEADS = 16
HEADS_PER_NGRAM = 8
NGRAM_SIZE = 3
FAKE_EOS = 999_999_999  # engraft/testing/fake_table.py:20

# Synthetic IQ4_NL table (the real table's format at a small size).
SYN_HEAD_SIZES = [1009, 1013, 1019, 1021, 1031, 1033, 1039, 1049,
                  2003, 2011, 2017, 2027, 2029, 2039, 2053, 2063]
SYN_EOS = 248044  # the corpus EOS of the real model
SYN_IMAGE_TOKEN = 248056
SYN_SEED = 20260901


def head_offsets(sizes):
    off, acc = [], 0
    for s in sizes:
        off.append(acc)
        acc += int(s)
    return off


def fake_table_params(seed: int = 0, head_vocab_size: int = 5_000) -> dict:
    """Addressing constants of FakeTable(seed, head_vocab_size), restating
    engraft/testing/fake_table.py:24-36 (four multipliers, odd, < 2**61)."""
    rng = np.random.default_rng(seed)
    mult = [int(rng.integers(1, 2**61)) | 1 for _ in range(NGRAM_SIZE + 1)]
    sizes = [head_vocab_size] * N_HEADS
    return dict(mult=mult, head_sizes=sizes, head_offsets=head_offsets(sizes), eos=FAKE_EOS,
                ngram_size=NGRAM_SIZE, hpn=HEADS_PER_NGRAM)


def fake_table_rows(seed: int = 0, head_vocab_size: int = 5_000) -> np.ndarray:
    """Every row of FakeTable(seed, head_vocab_size) in global-id order,
    float32 [16*p, 160] (engraft/testing/fake_table.py:70-76)."""
    p = head_vocab_size
    out = np.empty((N_HEADS * p, ROW_LEN), dtype=np.float32)
    for h in range(N_HEADS):
        for r in range(p):
            rng = np.random.default_rng((seed, h, r))
            out[h * p + r] = rng.standard_normal(ROW_LEN).astype(np.float32) * 0.05
    return out


def syn_params() -> dict:
    rng = np.random.default_rng(SYN_SEED)
    mult = [int(x) | 1 for x in rng.integers(0, 2**63, size=NGRAM_SIZE + 1, dtype=np.uint64)]
    mult[0] |= 1 << 63  # exercise products with the top bit set
    mult[2] |= 1 << 63
    return dict(mult=mult, head_sizes=list(SYN_HEAD_SIZES), head_offsets=head_offsets(SYN_HEAD_SIZES),
                eos=SYN_EOS, ngram_size=NGRAM_SIZE, hpn=HEADS_PER_NGRAM)


def _fp16_scales(rng, n, sigma):
    d = (rng.standard_normal(n) * sigma).astype(np.float16)
    return d


def iq4nl_raw(n_rows: int, seed: int, dim: int = ROW_LEN) -> np.ndarray:
    """uint8 [n_rows, dim/32*18]: per block an fp16 scale ~N(0, 1e-3) then 16
    random nibble bytes; a few special scales (0, -0, fp16 subnormal, large)."""
    rng = np.random.default_rng(seed)
    nb = dim // 32
    blocks = np.empty((n_rows, nb, 18), dtype=np.uint8)
    d = _fp16_scales(rng, n_rows * nb, 1e-3).reshape(n_rows, nb)
    flat = d.reshape(-1)
    specials = np.array([0.0, -0.0, 6e-8, 3e-5, 1000.0, -2.5], dtype=np.float16)
    k = min(len(specials), flat.size)
    flat[:k] = specials[:k]
    blocks[:, :, 0:2] = d.view(np.uint8).reshape(n_rows, nb, 2)
    blocks[:, :, 2:] = rng.integers(0, 256, size=(n_rows, nb, 16), dtype=np.uint8)
    if n_rows > 8:
        blocks[7, :, 0:2] = 0  # an all-zero-scale row (engraft/table.py:172-183)
    return blocks.reshape(n_rows, nb * 18)


def iq4xs_raw(n_rows: int, seed: int, dim: int = 256) -> np.ndarray:
    """uint8 [n_rows, dim/256*136]: per superblock fp16 d ~N(0, 1e-3), random
    scales_h (u16), scales_l (4 B) and qs (128 B)."""
    rng = np.random.default_rng(seed)
    ns = dim // 256
    sb = np.empty((n_rows, ns, 136), dtype=np.uint8)
    d = _fp16_scales(rng, n_rows * ns, 1e-3).reshape(n_rows, ns)
    sb[:, :, 0:2] = d.view(np.uint8).reshape(n_rows, ns, 2)
    sb[:, :, 2:] = rng.integers(0, 256, size=(n_rows, ns, 134), dtype=np.uint8)
    return sb.reshape(n_rows, ns * 136)


def syn_table_raw() -> np.ndarray:
    """Raw IQ4_NL bytes of the synthetic table, all heads in global-id order."""
    return iq4nl_raw(sum(SYN_HEAD_SIZES), seed=SYN_SEED + 1)


def synthetic_corpus(n: int, seed: int, eos: int, vocab: int = 50, every: int = 200) -> np.ndarray:
    """int32 tokens uniform over [0, vocab) with EOS every `every` tokens (the
    shape of the reference's own corpus in tests/test_damage.py:19-24)."""
    rng = np.random.default_rng(seed)
    tokens = rng.integers(0, vocab, size=n, dtype=np.int32)
    tokens[every - 1::every] = eos
    return tokens


def fragments(seed: int, n_frag: int, vocab: int, eos: int, lo: int = 3, hi: int = 30) -> list[list[int]]:
    """Random raw fragments (no leading EOS) for pack_fragments; one interior EOS."""
    rng = np.random.default_rng(seed)
    out = []
    for i in range(n_frag):
        ln = int(rng.integers(lo, hi))
        f = [int(x) for x in rng.integers(0, vocab, size=ln)]
        if i == 1 and ln > 4:
            f[2] = eos
        out.append(f)
    return out


def seg_starts(segment_ids) -> np.ndarray:
    """seg_start[i] = first index holding segment_ids[i]'s value: the
    reference's OverlayEmb.__post_init__ rule (engraft/replica/seq.py:317-335)."""
    seg = np.asarray(segment_ids, dtype=np.int64)
    first: dict[int, int] = {}
    out = np.empty(seg.shape[0], dtype=np.int32)
    for i, v in enumerate(seg.tolist()):
        if v not in first:
            first[v] = i
        out[i] = first[v]
    return out


def overlay_noise(seed: int, shape) -> np.ndarray:
    """Perturbation added to the true rows to make the overlay rows visible."""
    return (np.random.default_rng((seed, 1)).standard_normal(shape) * 0.01).astype(np.float32)


def overlay_grad(seed: int, shape) -> np.ndarray:
    """Upstream gradient fed to the overlay embedding's backward, ~N(0, 1e-3)."""
    return (np.random.default_rng((seed, 2)).standard_normal(shape) * 1e-3).astype(np.float32)


def pleo_fact(k: int, pool: np.ndarray, pool_true_rows: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Rows and data of the k-th synthetic .pleo "fact" over a pool of global
    rows (pool_true_rows[i] = true row of pool[i]): a seeded 40 % subset of the
    pool at its true values, with seeded noise added to about half of the rows
    (the others keep a delta of exactly zero).  Fact 1 lists its rows in a
    shuffled order."""
    rng = np.random.default_rng((k, 3))
    pick = np.sort(rng.choice(pool.size, size=max(1, pool.size * 2 // 5), replace=False))
    if k == 1:
        pick = pick[rng.permutation(pick.size)]
    rows = pool[pick].astype(np.int32)
    data = pool_true_rows[pick].astype(np.float32).copy()
    moved = rng.random(rows.size) < 0.5
    data[moved] += (rng.standard_normal((int(moved.sum()), data.shape[1])) * 0.01).astype(np.float32)
    return rows, data


def rowset_case_sets(all_read: np.ndarray) -> dict:
    """The census row lists of the row-set golden case, derived from all_read."""
    a = np.asarray(all_read, dtype=np.int64)
    return {"all_read": a.tolist(), "neutral_read": a[::3].tolist(), "entity": a[::5].tolist(),
            "terme": a[1::7].tolist(), "t8_answer": a[2::4].tolist()}


ROWSET_EXCLUDE = {0: [1, 2], 3: [0], 5: [4, 5, 6]}


# The PLE block (engraft/replica/layers.py:565-626) at reduced width: hc streams
# of n_embd channels, conv of K taps with dilation 3 (the n-gram size).
PLE_CASES = [  # (seed, T, history rows)
    (1, 11, 0),   # start of a sequence: empty history
    (2, 5, 9),    # a full history of (K-1)*dilation rows
    (3, 1, 9),    # one decode step
    (4, 4, 5),    # a history shorter than (K-1)*dilation
]
PLE_HC, PLE_N, PLE_K, PLE_DIL, PLE_EPS = 2, 256, 4, 3, 1e-6


def ple_case(seed: int, T: int, n_hist: int, hc: int = PLE_HC, n: int = PLE_N, K: int = PLE_K) -> dict:
    """Seeded inputs of one ple_forward call: emb [T, n], hidden [T, hc, n],
    hist [n_hist, hc, n], and the block's weights (norm weights near 1, the
    rest ~N(0, 0.1^2) as the reference's layer tests draw them)."""
    rng = np.random.default_rng(1000 + seed)
    f = lambda *s: (rng.standard_normal(s) * 0.1).astype(np.float32)  # noqa: E731
    return dict(emb=f(T, n), hidden=f(T, hc, n), hist=f(n_hist, hc, n), w_key=f(hc * n, n), w_value=f(n, n),
                norm_key=(1.0 + f(hc * n)).astype(np.float32), norm_query=(1.0 + f(hc * n)).astype(np.float32),
                norm_conv=(1.0 + f(hc * n)).astype(np.float32), conv1d=f(hc * n, K))
