"""The allocation-free sort entry point, gs_isect_sort_noalloc.

It exists for callers that may not allocate device memory while they run
(an engine that owns all device buffers and passes a plugin only its inputs
and outputs).  It must give exactly what the workspace-taking sort
(gs_isect_sort) gives, call after call, even though every call reuses the
same fixed scratch array inside the library.  This file is collected last so
that a failure here cannot hide the results of the other tests."""
from __future__ import annotations

import ctypes as ct

import numpy as np
import pytest
import torch

from _util import assert_exact

pytestmark = pytest.mark.gpu

MAX_ISECTS = 1 << 20


def _keys(n, bits, seed):
    rng = np.random.default_rng(seed)
    keys = (rng.integers(0, 1 << min(bits - 32, 20), size=n).astype(np.int64) << 32) | \
        rng.integers(0, 512, size=n).astype(np.int64)  # many duplicates: stability matters
    if bits == 64:
        keys |= rng.integers(0, 1 << 30, size=n).astype(np.int64) << 33
        neg = rng.uniform(size=n) < 0.5
        keys[neg] = -keys[neg]
    return keys, rng.permutation(n).astype(np.int32)


def test_noalloc_sort_matches_workspace_sort(gs, cuda):
    lib = gs.load()
    stream = ct.c_void_p(torch.cuda.current_stream().cuda_stream)
    # Calls in a row, small then the largest then small again: none may see
    # anything of the one before it in the shared scratch array.
    for n, bits, seed in ((300_001, 46, 1), (MAX_ISECTS, 64, 2), (5_000, 46, 3)):
        k, v = _keys(n, bits, seed)
        keys = torch.from_numpy(k).to(cuda)
        vals = torch.from_numpy(v).to(cuda)
        want_k, want_v = gs.intersect_tile_sort(keys, vals, bits)
        got_k = torch.empty_like(keys)
        got_v = torch.empty_like(vals)
        rc = lib.gs_isect_sort_noalloc(n, bits, ct.c_void_p(keys.data_ptr()),
                                       ct.c_void_p(vals.data_ptr()), ct.c_void_p(got_k.data_ptr()),
                                       ct.c_void_p(got_v.data_ptr()), stream)
        assert rc == 0, lib.gs_last_error()
        # no bounded wait of this sort gave up
        assert lib.gs_isect_sort_noalloc_check(n, stream) == 0, lib.gs_last_error()
        torch.cuda.synchronize()
        assert_exact(got_k, want_k, f"keys (n={n})")
        assert_exact(got_v, want_v, f"values (n={n})")
    # an empty sort launches nothing and succeeds
    assert lib.gs_isect_sort_noalloc(0, 46, None, None, None, None, stream) == 0
    assert lib.gs_isect_sort_noalloc_check(0, stream) == 0


def test_noalloc_sort_rejects_oversize(gs, cuda):
    lib = gs.load()
    rc = lib.gs_isect_sort_noalloc(MAX_ISECTS + 1, 46, None, None, None, None, None)
    assert rc == 1  # GS_ERR_INVALID, before any launch
    assert b"at most" in lib.gs_last_error()
