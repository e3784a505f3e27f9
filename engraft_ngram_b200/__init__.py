"""B200-native (sm_100a) Engram/PLE table path of ENGRAFT.

hash the last 2 and 3 tokens into 16 row ids -> gather the resident 4-bit (or
fp32) rows with the trainable overlay rows substituted -> dequantise -> emit;
backward: deterministic duplicate-reducing row gradients; then the fused Adam
step with the descent's regulariser.  All compute runs in hand-written CUDA
kernels behind the C ABI of include/engram_b200.h (libengram_b200.so); there is
no CPU fallback.

Drop-in use with the reference:
    import engraft_ngram_b200 as eb
    eb.install()            # engraft.replica.seq.OverlayEmb -> eb.OverlayEmb
"""
from __future__ import annotations

from . import _lib
from ._lib import FMT_F32, FMT_IQ4_NL, FMT_IQ4_XS, MODE_CONCAT_F32, MODE_PAIRSUM_ADD_BF16
from .optim import OverlayAdam, reg_scale
from .overlay import (OverlayEmb, OverlayMap, engram_embed, engram_embed_at, engram_residual_add, forget_overlay_map,
                      row_gradients, seg_starts_from_segment_ids)
from .patch import (install, install_ple, install_rowsets, install_scan, uninstall, uninstall_ple, uninstall_rowsets,
                    uninstall_scan)
from .ple import ple_forward
from .pleo import read_pleo, read_pleo_device, write_pleo
from .rowset import DeviceRowSet, build_all_read_row_set, build_rows_var, sum_overlays, write_merged_pleo
from .scan import scan_hits
from .table import DeviceTable

__all__ = [
    "DeviceTable", "OverlayEmb", "OverlayMap", "OverlayAdam", "engram_embed", "engram_embed_at", "engram_residual_add",
    "row_gradients", "seg_starts_from_segment_ids", "reg_scale", "install", "uninstall", "install_scan",
    "uninstall_scan", "install_rowsets", "uninstall_rowsets", "DeviceRowSet", "build_all_read_row_set",
    "build_rows_var", "sum_overlays", "write_merged_pleo", "read_pleo",
    "write_pleo", "read_pleo_device", "FMT_F32", "FMT_IQ4_NL", "FMT_IQ4_XS", "MODE_CONCAT_F32",
    "MODE_PAIRSUM_ADD_BF16", "load_library", "scan_hits", "ple_forward", "install_ple", "uninstall_ple",
    "forget_overlay_map",
]


def load_library():
    """Loads libengram_b200.so (raises if it has not been built)."""
    return _lib.load()
