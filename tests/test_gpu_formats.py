"""gs_spz_attributes (gsplat_core.formats.spz_attributes) on the GPU: every
scale / rotation / quaternion-order / colour mode against the reference's own
export_trained_spz output (tests/golden/formats.npz), and against the oracle
at a larger size.  fp32 arithmetic in the reference's operation order: within
1e-6 absolute (the vector norms may round differently from numpy's)."""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch

from oracle.formats import spz_attributes as oracle_spz
from test_formats import FIELDS, GOLDEN, _inputs

pytestmark = pytest.mark.gpu


def _run(means, q, ls, ol, col, rest, scale, rot, order, color, src, d):
    from gsplat_core import formats
    T = lambda x: torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()  # noqa: E731
    kw = dict(colors=T(col)) if src == "rgb" else dict(features_dc=T(col), features_rest=T(rest))
    return formats.spz_attributes(T(means), T(q), T(ls), T(ol), sh_degree=d, scale_mode=scale,
                                  rotation_mode=rot, quat_order=order, color_mode=color, **kw)


def test_spz_attributes_match_reference_export(cuda):
    g = np.load(os.path.join(GOLDEN, "formats.npz"))
    worst = 0.0
    for tag in (str(t) for t in g["cases"]):
        scale, rot, order, color, src, d = tag.split(".")
        out = _run(*_inputs(g, src), scale, rot, order, color, src, int(d))
        torch.cuda.synchronize()
        for f in FIELDS:
            a, e = out[f].cpu().numpy(), g[f"{tag}.{f}"]
            assert a.shape == e.shape, (tag, f)
            if e.size:
                worst = max(worst, float(np.abs(a - e).max()))
        assert out["sh_degree"] == int(g[f"{tag}.sh_degree"])
    assert worst <= 1e-6, worst


@pytest.mark.parametrize("rot", ["direct", "position_axis", "fastgs_conjugate",
                                 "position_conjugate"])
def test_spz_attributes_match_oracle_large(cuda, rot):
    rng = np.random.default_rng(4)
    n = 200_003
    means = rng.normal(size=(n, 3)).astype(np.float32)
    q = rng.normal(size=(n, 4)).astype(np.float32)
    q[:4] = [[1, 0, 0, 0], [0, 1, 0, 0], [0, 0, 1, 0], [0, 0, 0, 1]]
    ls = rng.uniform(-6, -1, size=(n, 3)).astype(np.float32)
    ol = rng.uniform(-6, 6, size=n).astype(np.float32)
    dc = rng.normal(size=(n, 3)).astype(np.float32)
    rest = rng.normal(size=(n, 15, 3)).astype(np.float32)
    out = _run(means, q, ls, ol, dc, rest, "scanner_axis", rot, "xyzw", "sh", "sh", 3)
    e = oracle_spz(means, q, ls, ol, dc, rest, "scanner_axis", rot, "xyzw", "sh", "sh", 3)
    for f in FIELDS:
        np.testing.assert_allclose(out[f].cpu().numpy(), np.asarray(e[f]).reshape(-1),
                                   rtol=0, atol=1e-6, err_msg=f)
