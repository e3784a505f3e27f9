"""Installs the CUDA path into the reference by monkeypatching, the reference's
own plugin idiom (engraft/replica/seq.py:1-17 shadows Replica attributes the
same way): engraft.replica.seq.OverlayEmb is looked up as a module global by
seq_forward (:907-909), seq_forward_triton (:1251-1253) and seq_step_triton
(:1430-1432), so replacing the module attribute reroutes every caller."""
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


def uninstall(seq_module=None):
    seq = seq_module or importlib.import_module("engraft.replica.seq")
    orig = _saved.get(id(seq), {}).pop("OverlayEmb", None)
    if orig is not None:
        seq.OverlayEmb = orig
    return seq
