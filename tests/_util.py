"""Comparison helpers shared by the tests."""
from __future__ import annotations

import numpy as np

# Tolerances of the parity contract: fp32 forward values within 1e-5
# absolute / 1e-4 relative; gradients within 1e-3 relative (atomic
# accumulation order differs from the sequential reference).
FWD_ATOL, FWD_RTOL = 1e-5, 1e-4
GRAD_RTOL = 1e-3


def to_np(x):
    try:
        import torch
        if isinstance(x, torch.Tensor):
            return x.detach().cpu().numpy()
    except ImportError:
        pass
    return np.asarray(x)


def assert_exact(actual, expected, what=""):
    a, e = to_np(actual), to_np(expected)
    assert a.shape == e.shape, f"{what}: shape {a.shape} != {e.shape}"
    if not np.array_equal(a, e):
        bad = np.flatnonzero(a.ravel() != e.ravel())
        raise AssertionError(f"{what}: {bad.size} of {a.size} entries differ, first at "
                             f"{bad[:5].tolist()}: {a.ravel()[bad[:5]]} vs {e.ravel()[bad[:5]]}")


def assert_fwd_close(actual, expected, what="", atol=FWD_ATOL, rtol=FWD_RTOL, mask=None):
    a, e = to_np(actual).astype(np.float64), to_np(expected).astype(np.float64)
    assert a.shape == e.shape, f"{what}: shape {a.shape} != {e.shape}"
    ok = np.abs(a - e) <= atol + rtol * np.abs(e)
    if mask is not None:
        ok |= ~np.broadcast_to(mask, ok.shape)
    if not ok.all():
        bad = np.flatnonzero(~ok.ravel())
        raise AssertionError(f"{what}: {bad.size} of {a.size} entries out of tolerance, max abs "
                             f"err {np.abs(a - e).max():.3e}; first {bad[:5].tolist()}: "
                             f"{a.ravel()[bad[:5]]} vs {e.ravel()[bad[:5]]}")


def assert_grad_close(actual, expected, what="", rtol=GRAD_RTOL, atol_frac=1e-5, noise=None,
                      noise_k=8.0):
    """|a - e| <= rtol |e| + atol_frac * max|e| (the absolute floor keeps
    entries that cancel to ~0 from failing on rounding alone).

    noise: |e - e'| with e' the same gradients summed in another order (the
    oracle run with another thread count).  Entries that are sums of many
    terms with heavy cancellation move by far more than 1e-3 of their value
    when only the order of the float additions changes; noise_k times that
    measured spread is added to their allowance."""
    a, e = to_np(actual).astype(np.float64), to_np(expected).astype(np.float64)
    assert a.shape == e.shape, f"{what}: shape {a.shape} != {e.shape}"
    scale = np.abs(e).max() if e.size else 0.0
    allow = rtol * np.abs(e) + atol_frac * scale + 1e-30
    if noise is not None:
        allow = allow + noise_k * np.abs(to_np(noise).astype(np.float64))
    ok = np.abs(a - e) <= allow
    if not ok.all():
        bad = np.flatnonzero(~ok.ravel())
        raise AssertionError(f"{what}: {bad.size} of {a.size} entries out of tolerance "
                             f"(scale {scale:.3e}); first {bad[:5].tolist()}: "
                             f"{a.ravel()[bad[:5]]} vs {e.ravel()[bad[:5]]}")
