"""Installs the CUDA path into the reference by monkeypatching, the reference's
own plugin idiom (engraft/replica/seq.py:1-17 shadows Replica attributes the
same way): engraft.replica.seq.OverlayEmb is looked up as a module global by
seq_forward (:907-909), seq_forward_triton (:1251-1253) and seq_step_triton
(:1430-1432), so replacing the module attribute reroutes every caller.
install_scan() does the same for engraft.damage.scan_hits (engraft/damage.py:168),
which the damage report calls as a module global, and install_rowsets() for the
row-set builders and overlay-file operations around the descent
(engraft.replica.distill.build_rows_var, engraft.descend_corpus's
build_all_read_row_set / write_merged_pleo / sum_overlays, and
engraft.replica.overlay_sum.sum_overlays)."""
from __future__ import annotations

import importlib

_saved: dict = {}


def install(seq_module=None):
    """Replaces engraft.replica.seq.OverlayEmb with engraft_ngram_b200.OverlayEmb.
    Returns the patched module."""
    from .overlay import OverlayEmb
    seq = seq_module or importlib.import_module("engraft.replica.seq")
    if "OverlayEmb" not in _saved.get(id(seq), {}):
        _saved.setdefault(id(seq), {})["OverlayEmb"] = seq.OverlayEmb
    seq.OverlayEmb = OverlayEmb
    return seq


def install_scan(damage_module=None):
    """Replaces engraft.damage.scan_hits with engraft_ngram_b200.scan_hits
    (same arguments; the corpus is hashed and scanned on the GPU)."""
    from .scan import scan_hits
    dmg = damage_module or importlib.import_module("engraft.damage")
    if "scan_hits" not in _saved.get(id(dmg), {}):
        _saved.setdefault(id(dmg), {})["scan_hits"] = dmg.scan_hits
    dmg.scan_hits = scan_hits
    return dmg


def uninstall_scan(damage_module=None):
    dmg = damage_module or importlib.import_module("engraft.damage")
    orig = _saved.get(id(dmg), {}).pop("scan_hits", None)
    if orig is not None:
        dmg.scan_hits = orig
    return dmg


_PLE_TARGETS = (("engraft.replica.layers", "ple_forward"), ("engraft.replica.model", "ple_forward"))


def install_ple(modules: dict | None = None) -> None:
    """Routes the reference's ple_forward (engraft/replica/layers.py:565-626, and
    the name engraft.replica.model imported) to engraft_ngram_b200.ple_forward,
    with or without gradients of emb, hidden and hist (the descent's backward
    through the block); calls that need gradients of the block's own weights,
    or whose tensors are not on a CUDA device, keep the reference's function.
    modules: name -> module overrides, for tests."""
    from . import ple
    for mod_name, attr in _PLE_TARGETS:
        mod = (modules or {}).get(mod_name) or importlib.import_module(mod_name)
        saved = _saved.setdefault(id(mod), {})
        if attr not in saved:
            saved[attr] = getattr(mod, attr)
        original = saved[attr]

        def routed(emb, hidden, w, hist, hparams, *args, _orig=original, **kw):
            if ple.weights_need_grad(w) or not emb.is_cuda:
                return _orig(emb, hidden, w, hist, hparams, *args, **kw)
            return ple.ple_forward(emb, hidden, w, hist, hparams, *args, **kw)

        setattr(mod, attr, routed)


def uninstall_ple(modules: dict | None = None) -> None:
    for mod_name, attr in _PLE_TARGETS:
        mod = (modules or {}).get(mod_name) or importlib.import_module(mod_name)
        orig = _saved.get(id(mod), {}).pop(attr, None)
        if orig is not None:
            setattr(mod, attr, orig)


_ROWSET_TARGETS = (
    ("engraft.replica.distill", "build_rows_var"),
    ("engraft.descend_corpus", "build_all_read_row_set"),
    ("engraft.descend_corpus", "write_merged_pleo"),
    ("engraft.descend_corpus", "sum_overlays"),
    ("engraft.replica.overlay_sum", "sum_overlays"),
)


def install_rowsets(modules: dict | None = None) -> None:
    """Replaces the row-set builders and overlay-file operations with their
    device versions (engraft_ngram_b200.rowset; same arguments and results).
    modules: {module name: module object} to patch instead of importing them."""
    from . import rowset
    for name, attr in _ROWSET_TARGETS:
        mod = (modules or {}).get(name) if modules is not None else importlib.import_module(name)
        if mod is None or not hasattr(mod, attr):
            continue
        saved = _saved.setdefault(id(mod), {})
        if attr not in saved:
            saved[attr] = getattr(mod, attr)
        setattr(mod, attr, getattr(rowset, attr))


def uninstall_rowsets(modules: dict | None = None) -> None:
    for name, attr in _ROWSET_TARGETS:
        mod = (modules or {}).get(name) if modules is not None else importlib.import_module(name)
        if mod is None:
            continue
        orig = _saved.get(id(mod), {}).pop(attr, None)
        if orig is not None:
            setattr(mod, attr, orig)


def uninstall(seq_module=None):
    seq = seq_module or importlib.import_module("engraft.replica.seq")
    orig = _saved.get(id(seq), {}).pop("OverlayEmb", None)
    if orig is not None:
        seq.OverlayEmb = orig
    return seq
