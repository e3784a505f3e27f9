"""CPU-only checks of the C-ABI library: it loads, exports every entry point
include/engram_b200.h declares, rejects bad arguments with the documented
status codes before touching the GPU, and its per-head division magic equals
Python's % on edge and random values."""
from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

import numpy as np
import pytest

import engraft_ngram_b200 as eb
from engraft_ngram_b200 import _lib as L

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def lib():
    from engraft_ngram_b200 import build
    build.build()
    return L.load()


def header_functions() -> list[str]:
    text = (ROOT / "include" / "engram_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:ENGRAM_API\s+)?(?:int|int64_t)\s+(engram_\w+)\s*\(", text, flags=re.M)))


def test_every_declared_symbol_is_exported(lib):
    names = header_functions()
    assert len(names) >= 12
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == set(L.SIGNATURES), "ctypes binding and header disagree"


def test_version_and_layout_helpers(lib):
    assert lib.engram_version() >= 100
    assert lib.engram_row_stride(L.FMT_F32, 128) == 512
    assert lib.engram_row_stride(L.FMT_IQ4_NL, 160) == 96
    assert lib.engram_row_stride(L.FMT_IQ4_XS, 256) == 144
    assert lib.engram_raw_row_bytes(L.FMT_IQ4_NL, 160) == 90
    assert lib.engram_raw_row_bytes(L.FMT_IQ4_XS, 256) == 136
    assert lib.engram_row_stride(L.FMT_IQ4_XS, 200) == L.ERR_FORMAT
    assert lib.engram_row_stride(L.FMT_F32, 2048) == L.ERR_FORMAT
    assert lib.engram_row_stride(7, 128) == L.ERR_FORMAT
    assert C.sizeof(L.EngramTable) == 8 * 3 + 4 * 6 + 8 + 8 * 4 + 8 * 32 + 4 * 32 * 2 + 8 * 32


def _init(lib, **kw):
    args = dict(rows=0x1000, n_rows=1000, fmt=L.FMT_F32, dim=128, ngram_size=3, hpn=8,
                sizes=[50] * 16, offs=[50 * h for h in range(16)], mult=[3, 5, 7, 9], eos=7)
    args.update(kw)
    t = L.EngramTable()
    s = np.asarray(args["sizes"], dtype=np.int64)
    o = np.asarray(args["offs"], dtype=np.int64)
    m = np.asarray(args["mult"], dtype=np.uint64)
    st = lib.engram_table_init(C.byref(t), args["rows"], args["n_rows"], args["fmt"], args["dim"],
                               args["ngram_size"], args["hpn"], s.ctypes.data, o.ctypes.data, m.ctypes.data,
                               len(m), args["eos"])
    return st, t


def test_table_init_validates(lib):
    st, t = _init(lib)
    assert st == 0 and t.n_heads == 16 and t.row_stride == 512 and t.head_size[3] == 50
    assert _init(lib, n_rows=0)[0] == L.ERR_RANGE
    assert _init(lib, offs=[50 * h + 1 for h in range(16)], n_rows=800)[0] == L.ERR_RANGE
    assert _init(lib, sizes=[0] + [50] * 15)[0] == L.ERR_RANGE
    assert _init(lib, rows=0x1004)[0] == L.ERR_ARG  # not 16-byte aligned
    assert _init(lib, ngram_size=5)[0] == L.ERR_ARG
    assert _init(lib, dim=100, fmt=L.FMT_IQ4_NL)[0] == L.ERR_FORMAT
    assert _init(lib, mult=[3, 5])[0] == L.ERR_ARG


def test_entry_points_reject_bad_arguments_without_launching(lib):
    st, t = _init(lib)
    ov = L.EngramOverlay(None, 0, None, None, 0)
    # negative sizes / null buffers / bad modes are rejected before any launch
    assert lib.engram_forward(C.byref(t), C.byref(ov), 0x1000, None, 0, -1, 0, 0x1000, None, None, None, None) == L.ERR_ARG
    assert lib.engram_forward(C.byref(t), C.byref(ov), None, None, 0, 5, 0, 0x1000, None, None, None, None) == L.ERR_ARG
    assert lib.engram_forward(C.byref(t), C.byref(ov), 0x1000, None, 0, 5, 9, 0x1000, None, None, None, None) == L.ERR_ARG
    assert lib.engram_forward(C.byref(t), C.byref(ov), 0x1000, None, 0, 5, 0, 0x1008, None, None, None, None) == L.ERR_ARG
    bad_ov = L.EngramOverlay(0x2000, 10, 0x3000, 0x4000, 12)  # capacity not a power of two
    assert lib.engram_forward(C.byref(t), C.byref(bad_ov), 0x1000, None, 0, 5, 0, 0x1000, None, None, None, None) == L.ERR_RANGE
    assert lib.engram_forward(C.byref(t), C.byref(ov), None, None, 0, 0, 0, None, None, None, None, None) == 0
    assert lib.engram_hash(C.byref(t), None, None, 0, 3, 0x1000, None) == L.ERR_ARG
    assert lib.engram_overlay_map_build(0x1000, 10, 0x2000, 0x3000, 16, None) == L.ERR_RANGE
    assert lib.engram_backward(0x1000, 10, 16, 8, 0, 0x2000, 128, 5, 0x3000, 0x4000, 0, None) == L.ERR_WORKSPACE
    assert lib.engram_backward(0x1000, 10, 16, 4, 1, 0x2000, 128, 5, 0x3000, 0x4000, 1 << 20, None) == L.ERR_FORMAT
    assert lib.engram_adam_step(0x1000, 0x1000, 0x1000, 0x1000, None, 10, 0, 1e-3, 0.9, 0.999, 1e-8, 0.0, None) == L.ERR_ARG
    assert lib.engram_backward_workspace_bytes(2048, 16, 40000) > 4 * 4 * 2048 * 16


def test_error_mapping():
    with pytest.raises(ValueError):
        L.check(L.ERR_RANGE, "x")
    with pytest.raises(RuntimeError):
        L.check(L.ERR_CUDA, "x")
    L.check(0, "x")


def test_division_magic_equals_python_mod(lib):
    rng = np.random.default_rng(0)
    divisors = [1, 2, 3, 7, 1 << 20, (1 << 20) + 1, 65521, 5000, 20_000_096, 2**31 - 1, 2**31 - 2,
                *[int(x) for x in rng.integers(1, 2**31, size=40)]]
    xs = np.concatenate([
        np.array([0, 1, 2, 2**63, 2**63 - 1, 2**64 - 1, 2**64 - 2, 2**32, 2**32 - 1], dtype=np.uint64),
        rng.integers(0, 2**64 - 1, size=20000, dtype=np.uint64, endpoint=True),
    ])
    out = np.empty_like(xs)
    for d in divisors:
        edge = np.array([d - 1, d, d + 1, 2 * d, (2**64 - 1) // d * d, (2**64 - 1) // d * d - 1],
                        dtype=np.uint64)
        x = np.concatenate([xs, edge])
        o = np.empty_like(x)
        assert lib.engram_selftest_mod(x.ctypes.data, len(x), d, o.ctypes.data) == 0
        assert np.array_equal(o, x % np.uint64(d)), d


def test_sharded_staged_and_ple_entry_points_reject_bad_arguments(lib):
    """The row-sharded, staging and PLE entry points refuse bad arguments with
    the documented codes before any launch (these calls never reach the GPU)."""
    st, t = _init(lib)
    assert st == 0
    ov = L.EngramOverlay(None, 0, None, None, 0)
    tok, seg, ptrs = 0x1000, 0x2000, 0x3000
    # engram_forward_sharded / engram_forward_staged
    assert lib.engram_forward_sharded(C.byref(t), C.byref(ov), tok, seg, -1, 5, ptrs, 2, 0, 0x4000, None, None,
                                      None, None) == L.ERR_ARG
    assert lib.engram_forward_sharded(C.byref(t), C.byref(ov), tok, seg, 0, 5, None, 2, 0, 0x4000, None, None,
                                      None, None) == L.ERR_ARG
    assert lib.engram_forward_staged(C.byref(t), C.byref(ov), tok, seg, 0, 5, ptrs, 2, 2, 0x5000, 0, 0x4000, None,
                                     None, None, None) == L.ERR_ARG  # rank outside the world
    assert lib.engram_forward_staged(C.byref(t), C.byref(ov), tok, seg, 0, 5, ptrs, 2, 0, None, 0, 0x4000, None,
                                     None, None, None) == L.ERR_ARG  # no stage with another rank's rows to read
    # pull staging
    assert lib.engram_stage_bytes(C.byref(t), 10) == 10 * 16 * 512
    assert lib.engram_stage_bytes(C.byref(t), -1) == L.ERR_ARG
    assert lib.engram_stage_sharded(C.byref(t), None, tok, seg, 0, 10, ptrs, 2, 0, 0x5008, 0, None) == L.ERR_ARG
    assert lib.engram_stage_sharded(C.byref(t), None, tok, seg, 0, 10, ptrs, 2, 0, 0x5000, -1, None) == L.ERR_ARG
    assert lib.engram_stage_sharded(C.byref(t), None, tok, seg, 0, 10, ptrs, 0, 0, 0x5000, 0, None) == L.ERR_ARG
    assert lib.engram_stage_sharded(C.byref(t), None, tok, seg, 0, 10, ptrs, 1, 0, 0x5000, 0, None) == 0  # one rank
    # push staging
    assert lib.engram_stage_plan_words(100, 2) == 2 * (4 + 1)
    assert lib.engram_stage_plan_words(-1, 2) == L.ERR_ARG
    assert lib.engram_stage_plan(C.byref(t), tok, seg, 0, 10, 17, 0x6000, 0x7000, None) == L.ERR_RANGE
    assert lib.engram_stage_plan(C.byref(t), None, seg, 0, 10, 2, 0x6000, 0x7000, None) == L.ERR_ARG
    assert lib.engram_stage_push(C.byref(t), ptrs, None, ptrs, 0, 10, ptrs, 2, 2, 0, None) == L.ERR_ARG
    assert lib.engram_stage_push(C.byref(t), ptrs, None, ptrs, 0, 10, ptrs, 17, 0, 0, None) == L.ERR_RANGE
    # the PLE block
    args = [0x1000, 2560 * 5, 0x2000, 2560 * 5, 0x3000, 0x4000, 0x5000, 0x6000]
    assert lib.engram_ple_gate(*args, 4, 9, 2560, 1e-6, 0x7000, None, 0x8000, None) == L.ERR_ARG  # hc > 8
    assert lib.engram_ple_gate(*args, 4, 4, 2562, 1e-6, 0x7000, None, 0x8000, None) == L.ERR_ARG  # n % 4
    bad = list(args)
    bad[0] = 0x1004
    assert lib.engram_ple_gate(*bad, 4, 4, 2560, 1e-6, 0x7000, None, 0x8000, None) == L.ERR_ARG  # misaligned key
    conv = [0x1000, 2560, 0x2000, 0x3000, 0x4000]
    assert lib.engram_ple_conv(*conv, None, 9, 0x5000, 4, 3, 4, 4, 2560, 0x6000, None) == L.ERR_ARG  # no history
    assert lib.engram_ple_conv(*conv, None, 0, 0x5000, 0, 3, 4, 4, 2560, 0x6000, None) == L.ERR_ARG  # K = 0
    assert lib.engram_ple_conv(*conv, None, 0, 0x5004, 4, 3, 4, 4, 2560, 0x6000, None) == L.ERR_ARG  # taps misaligned
    assert lib.engram_ple_conv(0x1000, 1 << 27, 0x2000, 0x3000, 0x4000, None, 0, 0x5000, 4, 3, 4, 8, 1 << 27,
                               0x6000, None) == L.ERR_RANGE  # hc * n too large for the kernel's indexing


def test_pushed_exchange_gemm_and_accumulate_entry_points_reject_bad_arguments(lib):
    """The pushed row exchange, the tcgen05 GEMMs and the ordered overlay
    accumulation refuse bad arguments with the documented codes before any
    CUDA call (these calls never reach the GPU)."""
    st, t = _init(lib)
    assert st == 0
    ov = L.EngramOverlay(None, 0, None, None, 0)
    tok, seg, idp, cnp, cnt, rix = 0x1000, 0x2000, 0x3000, 0x4000, 0x5000, 0x6000
    # engram_shard_route_push: n = 10 positions x 16 heads = 160 entries
    assert lib.engram_shard_route_push(None, C.byref(ov), tok, seg, 0, 10, 2, 0, idp, cnp, 160, cnt, rix,
                                       None) == L.ERR_ARG
    assert lib.engram_shard_route_push(C.byref(t), C.byref(ov), tok, seg, 0, 10, 2, 2, idp, cnp, 160, cnt, rix,
                                       None) == L.ERR_ARG  # rank outside the world
    assert lib.engram_shard_route_push(C.byref(t), C.byref(ov), tok, seg, 0, 10, 2, 0, None, cnp, 160, cnt, rix,
                                       None) == L.ERR_ARG  # no request buffers
    assert lib.engram_shard_route_push(C.byref(t), C.byref(ov), tok, seg, 0, 10, 2, 0, idp, cnp, 159, cnt, rix,
                                       None) == L.ERR_RANGE  # a region smaller than the batch
    assert lib.engram_shard_route_push(C.byref(t), C.byref(ov), tok, seg, 0, 10, 64, 0, idp, cnp, 1 << 26, cnt, rix,
                                       None) == L.ERR_RANGE  # world x region beyond the int32 row tags
    # engram_shard_serve_pushed
    shard, ids, counts, send = 0x10000, 0x20000, 0x30000, 0x40000
    assert lib.engram_shard_serve_pushed(shard, 144, 100, 0, 0, ids, counts, 160, send, None) == L.ERR_ARG
    assert lib.engram_shard_serve_pushed(shard, 136, 100, 2, 0, ids, counts, 160, send, None) == L.ERR_ARG  # stride % 16
    assert lib.engram_shard_serve_pushed(shard, 144, 100, 2, 0, ids, counts, 160, send + 8, None) == L.ERR_ARG
    assert lib.engram_shard_serve_pushed(shard, 144, 100, 2, 0, None, counts, 160, send, None) == L.ERR_ARG
    assert lib.engram_shard_serve_pushed(shard, 144, 100, 1, 0, ids, counts, 160, send, None) == 0  # one rank
    # engram_gemm_3xtf32 / engram_gemm_tf32
    a, b, c = 0x100000, 0x200000, 0x300000
    assert lib.engram_gemm_3xtf32(a, a, b, b, 128, 256, 30, 30, 30, c, 256, None, None) == L.ERR_ARG  # K % 4
    assert lib.engram_gemm_3xtf32(a, a, b, b, 128, 256, 32, 16, 32, c, 256, None, None) == L.ERR_ARG  # lda < K
    assert lib.engram_gemm_3xtf32(a + 4, a, b, b, 128, 256, 32, 32, 32, c, 256, None, None) == L.ERR_ARG
    assert lib.engram_gemm_3xtf32(a, a, b, b, 128, 256, 32, 32, 32, None, 256, None, None) == L.ERR_ARG
    assert lib.engram_gemm_3xtf32(a, a, b, b, 0, 256, 32, 32, 32, c, 256, None, None) == 0  # empty output
    ptrs = (C.c_void_p * 4)(a, a, a, a)
    assert lib.engram_gemm_tf32(0, ptrs, ptrs, 128, 256, 32, 32, 32, c, 256, None, None) == L.ERR_ARG
    assert lib.engram_gemm_tf32(4, ptrs, ptrs, 128, 256, 32, 32, 32, c, 256, None, None) == L.ERR_ARG
    # engram_overlay_accumulate (with and without the stable order of the targets)
    acc, index, order, data, base = 0x400000, 0x500000, 0x600000, 0x700000, 0x800000
    assert lib.engram_overlay_accumulate(acc, index, order, data, base, -1, 160, None) == L.ERR_ARG
    assert lib.engram_overlay_accumulate(acc, index, order, data, base, 10, 0, None) == L.ERR_ARG
    assert lib.engram_overlay_accumulate(None, index, order, data, base, 10, 160, None) == L.ERR_ARG
    assert lib.engram_overlay_accumulate(acc, index, None, data, base, 0, 160, None) == 0  # nothing to add
