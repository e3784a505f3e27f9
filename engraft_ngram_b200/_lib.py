"""ctypes binding of libengram_b200.so (the C ABI declared in include/engram_b200.h).

The reference is Python, so ctypes is the FFI it would bind; this module is
that binding.  There is no fallback: if the library is missing or cannot be
loaded, importing the package's compute entry points raises.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("ENGRAM_B200_LIB", PKG / "libengram_b200.so"))

OK, ERR_ARG, ERR_FORMAT, ERR_RANGE, ERR_WORKSPACE, ERR_CUDA = 0, -1, -2, -3, -4, -5
FMT_F32, FMT_IQ4_NL, FMT_IQ4_XS = 0, 1, 2
MODE_CONCAT_F32, MODE_PAIRSUM_ADD_BF16 = 0, 1
MAX_HEADS, MAX_CTX = 32, 4

FMT_NAMES = {"f32": FMT_F32, "iq4_nl": FMT_IQ4_NL, "iq4_xs": FMT_IQ4_XS}

_ERR_TEXT = {
    ERR_ARG: "invalid argument (null pointer, negative size, misaligned buffer or bad enum)",
    ERR_FORMAT: "unsupported format / dim / mode combination",
    ERR_RANGE: "value out of range",
    ERR_WORKSPACE: "workspace too small",
    ERR_CUDA: "CUDA launch failed",
}


class EngramTable(C.Structure):
    _fields_ = [
        ("rows", C.c_void_p),
        ("n_rows", C.c_int64),
        ("row_stride", C.c_int64),
        ("fmt", C.c_int32),
        ("dim", C.c_int32),
        ("ngram_size", C.c_int32),
        ("heads_per_ngram", C.c_int32),
        ("n_heads", C.c_int32),
        ("reserved", C.c_int32),
        ("eos_token_id", C.c_int64),
        ("mult", C.c_uint64 * MAX_CTX),
        ("head_magic", C.c_uint64 * MAX_HEADS),
        ("head_size", C.c_uint32 * MAX_HEADS),
        ("head_shift", C.c_uint32 * MAX_HEADS),
        ("head_offset", C.c_int64 * MAX_HEADS),
    ]


class EngramOverlay(C.Structure):
    _fields_ = [
        ("rows", C.c_void_p),
        ("n_rows", C.c_int64),
        ("map_keys", C.c_void_p),
        ("map_slots", C.c_void_p),
        ("capacity", C.c_int64),
    ]


# name -> (restype, argtypes); the single source of the exported symbol list
SIGNATURES = {
    "engram_version": (C.c_int, []),
    "engram_row_stride": (C.c_int64, [C.c_int32, C.c_int32]),
    "engram_raw_row_bytes": (C.c_int64, [C.c_int32, C.c_int32]),
    "engram_table_init": (C.c_int, [C.POINTER(EngramTable), C.c_void_p, C.c_int64, C.c_int32, C.c_int32, C.c_int32,
                                    C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int32, C.c_int64]),
    "engram_table_pack": (C.c_int, [C.c_int32, C.c_int32, C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p]),
    "engram_overlay_map_build": (C.c_int, [C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p, C.c_int64, C.c_void_p]),
    "engram_overlay_lookup": (C.c_int, [C.POINTER(EngramOverlay), C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p]),
    "engram_hash": (C.c_int, [C.POINTER(EngramTable), C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.c_void_p,
                              C.c_void_p]),
    "engram_forward": (C.c_int, [C.POINTER(EngramTable), C.POINTER(EngramOverlay), C.c_void_p, C.c_void_p, C.c_int64,
                                 C.c_int64, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "engram_forward_at": (C.c_int, [C.POINTER(EngramTable), C.POINTER(EngramOverlay), C.c_void_p, C.c_int64,
                                    C.c_void_p, C.c_void_p, C.c_int64, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p,
                                    C.c_void_p, C.c_void_p]),
    "engram_forward_indirect": (C.c_int, [C.POINTER(EngramTable), C.POINTER(EngramOverlay), C.c_void_p, C.c_void_p,
                                          C.c_int64, C.c_int64, C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p,
                                          C.c_void_p, C.c_void_p, C.c_void_p]),
    "engram_shard_requests": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int64, C.c_int32, C.c_void_p, C.c_void_p,
                                        C.c_int64, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "engram_shard_plan": (C.c_int, [C.POINTER(EngramTable), C.POINTER(EngramOverlay), C.c_void_p, C.c_void_p,
                                    C.c_int64, C.c_int64, C.c_int32, C.c_int32, C.c_void_p, C.c_void_p, C.c_int64,
                                    C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "engram_forward_exchanged": (C.c_int, [C.POINTER(EngramTable), C.POINTER(EngramOverlay), C.c_void_p, C.c_void_p,
                                           C.c_int64, C.c_int64, C.c_void_p, C.c_int32, C.c_int32, C.c_void_p,
                                           C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                           C.c_void_p]),
    "engram_shard_route_scratch_words": (C.c_int64, [C.c_int64, C.c_int32, C.c_int32]),
    "engram_shard_route": (C.c_int, [C.POINTER(EngramTable), C.POINTER(EngramOverlay), C.c_void_p, C.c_void_p,
                                     C.c_int64, C.c_int64, C.c_int32, C.c_int32, C.c_void_p, C.c_int64, C.c_void_p,
                                     C.c_void_p, C.c_void_p, C.c_void_p]),
    "engram_shard_route_push": (C.c_int, [C.POINTER(EngramTable), C.POINTER(EngramOverlay), C.c_void_p,
                                          C.c_void_p, C.c_int64, C.c_int64, C.c_int32, C.c_int32, C.c_void_p,
                                          C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p, C.c_void_p]),
    "engram_shard_serve_pushed": (C.c_int, [C.c_void_p, C.c_int64, C.c_int64, C.c_int32, C.c_int32, C.c_void_p,
                                            C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p]),
    "engram_shard_gather": (C.c_int, [C.c_void_p, C.c_int64, C.c_int64, C.c_void_p, C.c_int64, C.c_int32, C.c_void_p,
                                      C.c_void_p]),
    "engram_gather_rows": (C.c_int, [C.POINTER(EngramTable), C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p]),
    "engram_backward_workspace_bytes": (C.c_int64, [C.c_int64, C.c_int32, C.c_int64]),
    "engram_backward": (C.c_int, [C.c_void_p, C.c_int64, C.c_int32, C.c_int32, C.c_int32, C.c_void_p, C.c_int32,
                                  C.c_int64, C.c_void_p, C.c_void_p, C.c_int64, C.c_void_p]),
    "engram_backward_noalloc": (C.c_int, [C.c_void_p, C.c_int64, C.c_int32, C.c_int32, C.c_int32, C.c_void_p,
                                          C.c_int32, C.c_int64, C.c_void_p, C.c_void_p]),
    "engram_adam_step": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int64,
                                   C.c_double, C.c_double, C.c_double, C.c_double, C.c_float, C.c_void_p]),
    "engram_scan_hits_workspace_bytes": (C.c_int64, [C.c_int64]),
    "engram_scan_hits": (C.c_int, [C.POINTER(EngramTable), C.c_void_p, C.c_int64, C.c_int64, C.c_int64, C.c_int32,
                                   C.POINTER(EngramOverlay), C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                   C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_void_p]),
    "engram_rowset_words": (C.c_int64, [C.c_int64]),
    "engram_rowset_mark": (C.c_int, [C.POINTER(EngramTable), C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p,
                                     C.c_int64, C.c_void_p, C.c_void_p]),
    "engram_rowset_mark_ids": (C.c_int, [C.c_void_p, C.c_int64, C.c_int64, C.c_void_p, C.c_void_p]),
    "engram_rowset_combine": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int64, C.c_int32, C.c_void_p, C.c_void_p]),
    "engram_rowset_workspace_bytes": (C.c_int64, [C.c_int64]),
    "engram_rowset_extract": (C.c_int, [C.c_void_p, C.c_int64, C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p,
                                        C.c_int64, C.c_void_p]),
    "engram_rowset_index": (C.c_int, [C.c_void_p, C.c_int64, C.c_void_p, C.c_int64, C.c_void_p, C.c_int64,
                                      C.c_void_p, C.c_void_p]),
    "engram_overlay_accumulate": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64,
                                            C.c_int32, C.c_void_p]),
    "engram_backward_to_owners": (C.c_int, [C.c_void_p, C.c_int64, C.c_int32, C.c_int32, C.c_int32, C.c_void_p,
                                            C.c_int32, C.c_int64, C.c_void_p, C.c_int32, C.c_int32, C.c_void_p,
                                            C.c_int64, C.c_void_p]),
    "engram_adam_owner_step": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int32, C.c_int32, C.c_int64, C.c_int32,
                                         C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_double, C.c_double,
                                         C.c_double, C.c_double, C.c_float, C.c_void_p]),
    "engram_forward_sharded": (C.c_int, [C.POINTER(EngramTable), C.POINTER(EngramOverlay), C.c_void_p, C.c_void_p,
                                         C.c_int64, C.c_int64, C.c_void_p, C.c_int32, C.c_int32, C.c_void_p,
                                         C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "engram_stage_bytes": (C.c_int64, [C.POINTER(EngramTable), C.c_int64]),
    "engram_stage_sharded": (C.c_int, [C.POINTER(EngramTable), C.POINTER(EngramOverlay), C.c_void_p, C.c_void_p,
                                       C.c_int64, C.c_int64, C.c_void_p, C.c_int32, C.c_int32, C.c_void_p, C.c_int32,
                                       C.c_void_p]),
    "engram_stage_plan_words": (C.c_int64, [C.c_int64, C.c_int32]),
    "engram_stage_plan": (C.c_int, [C.POINTER(EngramTable), C.c_void_p, C.c_void_p, C.c_int64, C.c_int64,
                                    C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p]),
    "engram_stage_push": (C.c_int, [C.POINTER(EngramTable), C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64,
                                    C.c_int64, C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_void_p]),
    "engram_forward_staged": (C.c_int, [C.POINTER(EngramTable), C.POINTER(EngramOverlay), C.c_void_p, C.c_void_p,
                                        C.c_int64, C.c_int64, C.c_void_p, C.c_int32, C.c_int32, C.c_void_p,
                                        C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "engram_gemm_tf32": (C.c_int, [C.c_int32, C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.c_int64, C.c_int64,
                                   C.c_int64, C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p]),
    "engram_gemm_3xtf32": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int64,
                                     C.c_int64, C.c_int64, C.c_int64, C.c_void_p, C.c_int64, C.c_void_p,
                                     C.c_void_p]),
    "engram_ple_gate_backward": (C.c_int, [C.c_void_p, C.c_int64, C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p,
                                           C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                           C.c_int64, C.c_int32, C.c_int32, C.c_float, C.c_int32, C.c_int32,
                                           C.c_void_p, C.c_int64, C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p]),
    "engram_ple_conv_backward": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int64, C.c_void_p, C.c_int32, C.c_int32,
                                           C.c_int64, C.c_int32, C.c_int32, C.c_void_p, C.c_void_p, C.c_int64,
                                           C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "engram_ple_gate": (C.c_int, [C.c_void_p, C.c_int64, C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p,
                                  C.c_void_p, C.c_void_p, C.c_int64, C.c_int32, C.c_int32, C.c_float, C.c_void_p,
                                  C.c_void_p, C.c_void_p, C.c_void_p]),
    "engram_ple_conv": (C.c_int, [C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                  C.c_int64, C.c_void_p, C.c_int32, C.c_int32, C.c_int64, C.c_int32, C.c_int32,
                                  C.c_void_p, C.c_void_p]),
    "engram_selftest_mod": (C.c_int, [C.c_void_p, C.c_int64, C.c_uint32, C.c_void_p]),
    "engram_launch_count": (C.c_int64, []),
}

_lib = None


def load():
    """Loads the library once; raises if it is missing (no fallback path exists)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"libengram_b200.so not found at {LIB_PATH}: build it with "
                "`python -m engraft_ngram_b200.build` (nvcc, sm_100a); there is no CPU fallback")
        lib = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def check(status: int, what: str) -> None:
    """Maps a negative status to the exception the reference raises for it:
    ValueError for bad inputs (the reference's precondition errors,
    engraft/replica/pack.py:106-113), RuntimeError for a failed launch."""
    if status == OK:
        return
    msg = f"{what}: {_ERR_TEXT.get(status, 'error')} (status {status})"
    if status == ERR_CUDA:
        raise RuntimeError(msg)
    raise ValueError(msg)


def stream_of(device) -> int:
    import torch
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t) -> int | None:
    return None if t is None else t.data_ptr()
