"""engram_backward_noalloc: row gradients for callers that cannot allocate
device memory at the point they need them (an engine that reserves all GPU
memory up front, or code that must not take cudaMalloc's device-wide sync).

It must return exactly what engram_backward returns with a caller-provided
workspace.  Two calls in a row check that the library's shared scratch array
carries nothing from one call into the next; an over-limit size must be
refused before anything is launched.  The file sorts last so that a run which
stops at the first failure has run every other test first.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _case(seed, n, n_heads, R, dim, mode):
    rng = np.random.default_rng(seed)
    slots = np.where(rng.random((n, n_heads)) < 0.6, rng.integers(0, R, size=(n, n_heads)), -1).astype(np.int32)
    slots[:, 1] = np.where(rng.random(n) < 0.5, 3, slots[:, 1])  # a heavily duplicated row
    if mode == 0:
        grad = torch.from_numpy((rng.standard_normal((n, n_heads, dim)) * 1e-3).astype(np.float32))
    else:
        grad = torch.from_numpy(rng.standard_normal((n, n_heads // 2 * dim)).astype(np.float32) * 1e-2)
        grad = grad.to(torch.bfloat16)
    return torch.from_numpy(slots).to(DEV), grad.to(DEV)


def test_noalloc_backward_matches_workspace_backward_twice():
    if not torch.cuda.is_available():
        pytest.fail("needs a CUDA device")
    from engraft_ngram_b200 import _lib as L
    lib = L.load()
    stream = torch.cuda.current_stream().cuda_stream
    cases = [(1, 3000, 16, 70_000, 128, 0), (2, 1500, 16, 900, 256, 1)]  # second call: smaller, other mode
    for seed, n, nh, R, dim, mode in cases:
        slots, grad = _case(seed, n, nh, R, dim, mode)
        ws_bytes = int(lib.engram_backward_workspace_bytes(n, nh, R))
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=DEV)
        want = torch.full((R, dim), float("nan"), device=DEV)
        got = torch.full((R, dim), float("nan"), device=DEV)
        st = lib.engram_backward(slots.data_ptr(), n, nh, 8, mode, grad.data_ptr(), dim, R, want.data_ptr(),
                                 ws.data_ptr(), ws_bytes, stream)
        assert st == L.OK
        st = lib.engram_backward_noalloc(slots.data_ptr(), n, nh, 8, mode, grad.data_ptr(), dim, R,
                                         got.data_ptr(), stream)
        assert st == L.OK
        torch.cuda.synchronize()
        # the row gradients are bit-exact everywhere in this suite
        assert torch.equal(got.view(torch.int32), want.view(torch.int32)), (seed, mode)


def test_noalloc_backward_refuses_sizes_beyond_its_scratch():
    from engraft_ngram_b200 import _lib as L
    lib = L.load()
    n, nh, R = 1_000_000, 16, 40_000
    assert lib.engram_backward_workspace_bytes(n, nh, R) > 12 << 20
    # refused by the size check, before any pointer is used or any kernel launched
    st = lib.engram_backward_noalloc(0x1000, n, nh, 8, 0, 0x2000, 128, R, 0x3000, None)
    assert st == L.ERR_WORKSPACE
