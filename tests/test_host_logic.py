"""Host-side logic of the product package (no GPU): segment starts, row_map
validation, .pleo files, the install seam."""
from __future__ import annotations

import sys
import types

import numpy as np
import pytest
import torch

import fixtures as FX
import engraft_ngram_b200 as eb
from engraft_ngram_b200.overlay import OverlayMap


@pytest.mark.parametrize("seed", range(5))
def test_seg_starts_match_reference_rule(seed):
    rng = np.random.default_rng(seed)
    seg = np.sort(rng.integers(0, 20, size=500))
    if seed == 4:  # non-contiguous repeats follow the reference's first-occurrence rule
        seg = rng.integers(0, 6, size=300)
    assert np.array_equal(eb.seg_starts_from_segment_ids(torch.from_numpy(seg)), FX.seg_starts(seg))
    assert eb.seg_starts_from_segment_ids(np.zeros(0, np.int64)).shape == (0,)


def test_packed_segment_ids_example():
    # engraft/replica/pack.py example from the reference's tests/test_seq.py:55
    seg = torch.tensor([0, 0, 0, 0, 0, 1, 1, 1])
    assert eb.seg_starts_from_segment_ids(seg).tolist() == [0, 0, 0, 0, 0, 5, 5, 5]


def test_row_map_validation():
    with pytest.raises(NotImplementedError):
        OverlayMap.from_row_map({((1, 2, 3), 0): 0}, "cpu")
    with pytest.raises(ValueError):
        OverlayMap.from_row_map({5: 0, 6: 2}, "cpu")
    with pytest.raises(ValueError):
        OverlayMap.from_row_map({-3: 0}, "cpu")
    with pytest.raises(ValueError):
        OverlayMap.from_row_map({2**31: 0}, "cpu")


def test_pleo_bytes_identical_to_reference(golden, tmp_path):
    p = tmp_path / "x.pleo"
    eb.write_pleo(p, golden["pleo_rows"], golden["pleo_data"], strict_160=True)
    assert np.array_equal(np.frombuffer(p.read_bytes(), dtype=np.uint8), golden["pleo_bytes"])
    rows, data = eb.read_pleo(p)
    assert np.array_equal(rows, golden["pleo_rows"]) and np.array_equal(data, golden["pleo_data"])


def test_pleo_rejects_bad_magic_and_shapes(tmp_path):
    p = tmp_path / "bad.pleo"
    p.write_bytes(b"XXXX" + b"\0" * 8)
    with pytest.raises(ValueError):
        eb.read_pleo(p)
    with pytest.raises(ValueError):
        eb.write_pleo(tmp_path / "a.pleo", np.zeros(2, np.int32), np.zeros((2, 128), np.float32), strict_160=True)
    eb.write_pleo(tmp_path / "b.pleo", np.array([9, 3], np.int32), np.ones((2, 256), np.float32))
    rows, data = eb.read_pleo(tmp_path / "b.pleo")
    assert data.shape == (2, 256) and rows.tolist() == [9, 3]


def test_install_replaces_module_attribute():
    seq = types.SimpleNamespace(OverlayEmb="reference-class")
    eb.install(seq)
    assert seq.OverlayEmb is eb.OverlayEmb
    eb.uninstall(seq)
    assert seq.OverlayEmb == "reference-class"


def test_install_scan_replaces_module_attribute():
    dmg = types.SimpleNamespace(scan_hits="reference-function")
    eb.install_scan(dmg)
    assert dmg.scan_hits is eb.scan_hits
    eb.uninstall_scan(dmg)
    assert dmg.scan_hits == "reference-function"


def test_install_rowsets_replaces_and_restores_the_builders():
    names = ("engraft.replica.distill", "engraft.descend_corpus", "engraft.replica.overlay_sum")
    mods = {n: types.SimpleNamespace() for n in names}
    mods["engraft.replica.distill"].build_rows_var = "ref-brv"
    mods["engraft.descend_corpus"].build_all_read_row_set = "ref-ars"
    mods["engraft.descend_corpus"].write_merged_pleo = "ref-wmp"
    mods["engraft.descend_corpus"].sum_overlays = "ref-so"
    mods["engraft.replica.overlay_sum"].sum_overlays = "ref-so2"
    eb.install_rowsets(mods)
    assert mods["engraft.replica.distill"].build_rows_var is eb.build_rows_var
    assert mods["engraft.descend_corpus"].build_all_read_row_set is eb.build_all_read_row_set
    assert mods["engraft.descend_corpus"].write_merged_pleo is eb.write_merged_pleo
    assert mods["engraft.descend_corpus"].sum_overlays is eb.sum_overlays
    assert mods["engraft.replica.overlay_sum"].sum_overlays is eb.sum_overlays
    eb.uninstall_rowsets(mods)
    assert mods["engraft.replica.distill"].build_rows_var == "ref-brv"
    assert mods["engraft.replica.overlay_sum"].sum_overlays == "ref-so2"


def test_fragment_layout_of_the_row_set_builder():
    from engraft_ngram_b200.rowset import _fragments
    tokens, seg, pos = _fragments([[5, 6, 7], [8], [9, 10]])
    assert tokens.tolist() == [5, 6, 7, 8, 9, 10]
    assert seg.tolist() == [0, 0, 0, 3, 4, 4]
    assert pos.tolist() == [0, 1, 4]  # positions 0..len-2 of each fragment


def test_overlay_emb_refuses_cpu_tensors():
    ov = eb.OverlayEmb(object(), [1, 2, 3], torch.zeros(0, 160), {})
    with pytest.raises(RuntimeError):
        ov.build(3)


def test_bench_command_line_and_config_text(monkeypatch):
    """bench.py parses its flags and names the multi-GPU layout it ran
    (replicated, row-sharded with the deduplicated exchange (the default),
    staged row-sharded, in-place row-sharded, NCCL row-sharded)."""
    import bench
    monkeypatch.setattr(sys, "argv", ["bench.py", "--gpus", "2", "--shard", "--stage-blocks", "32"])
    args = bench.parse()
    assert args.shard and args.stage == "exchange" and args.stage_blocks == 32 and args.shard_exchange == "peer"
    assert args.e2e_exchange == "peer" and args.layout == "sharded"
    assert "three batches ahead" in bench.shard_text(dict(bench.CONFIGS["cfg5"], shard=True, stage="exchange"))
    cfg = dict(bench.CONFIGS["cfg5"], shard=True, shard_exchange="peer", stage="push", exchange="peer")
    text = bench.config_json(cfg, args)["parallelism"]
    assert text.startswith("dp2+row-sharded") and "stores the rows" in text
    assert "loaded from their owners" in bench.shard_text(dict(cfg, stage="pull"))
    assert "inside the forward" in bench.shard_text(dict(cfg, stage="off"))
    assert "NCCL all-to-all" in bench.shard_text(dict(cfg, shard_exchange="nccl"))
    assert bench.shard_text(dict(cfg, shard=False)) == ""


def test_tf32_split_is_exact():
    """split_tf32: hi keeps 10 explicit mantissa bits (low 13 bits zero) and
    hi + lo reproduces x exactly, for normal, tiny, huge and signed values."""
    from engraft_ngram_b200.ple import split_tf32
    g = torch.Generator().manual_seed(0)
    x = torch.cat([torch.randn(1000, generator=g), torch.randn(100, generator=g) * 1e-30,
                   torch.randn(100, generator=g) * 1e30, torch.tensor([0.0, -0.0, 1.0, -3.5])])
    hi, lo = split_tf32(x)
    assert torch.equal((hi.view(torch.int32) & 8191), torch.zeros_like(x, dtype=torch.int32))
    assert torch.equal(hi + lo, x)
    assert (lo.abs() <= x.abs() * 2.0 ** -10).all()


def test_overlay_map_cache_is_found_by_identity_and_size(monkeypatch):
    """OverlayEmb.build finds the device map of the same row_map dict without a
    pass over its items; a size change or forget_overlay_map rebuilds it."""
    from engraft_ngram_b200 import overlay as ov
    built = []

    class FakeMap:
        def __init__(self, rm):
            self.R = len(rm)

    monkeypatch.setattr(ov.OverlayMap, "from_row_map", classmethod(lambda cls, rm, dev: built.append(1) or FakeMap(rm)))
    ov.forget_overlay_map()
    rm = {10: 0, 20: 1}
    a = ov._overlay_map_for(rm, "cuda:0")
    assert ov._overlay_map_for(rm, "cuda:0") is a and len(built) == 1
    rm[30] = 2  # size changed: rebuilt
    b = ov._overlay_map_for(rm, "cuda:0")
    assert b is not a and b.R == 3 and len(built) == 2
    ov.forget_overlay_map(rm)
    assert ov._overlay_map_for(rm, "cuda:0") is not b and len(built) == 3
    assert ov._overlay_map_for(rm, "cuda:1") is not None and len(built) == 4  # one map per device
    pre = FakeMap({1: 0})
    pre.__class__ = type("M", (ov.OverlayMap,), {})  # an OverlayMap passed as row_map is used as it is
    assert ov._overlay_map_for(pre, "cuda:0") is pre
    ov.forget_overlay_map()
