"""Shared fixtures.  `-m gpu` tests need a CUDA device and call the product
through its C ABI; everything else runs on CPU (oracle against the golden
fixtures, the ABI surface, host-side validation, gloo multi-rank logic)."""
from __future__ import annotations

import os
import subprocess
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "gsplat-mlx_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (runs the sm_100a kernels)")


def _ensure_oracle():
    so = os.path.join(ROOT, "oracle", "liboracle.so")
    src = os.path.join(ROOT, "oracle", "gsplat_oracle.c")
    if not os.path.exists(so) or os.path.getmtime(so) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), "oracle"], check=True)


@pytest.fixture(scope="session")
def oracle():
    _ensure_oracle()
    from oracle.oracle import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def golden():
    def load(name):
        with np.load(os.path.join(GOLDEN, name + ".npz")) as d:
            return {k: d[k] for k in d.files}
    cache = {}

    def get(name):
        if name not in cache:
            cache[name] = load(name)
        return cache[name]
    return get


@pytest.fixture(scope="session")
def gs():
    """The product package, with its native library loaded."""
    import gsplat_core
    gsplat_core.load()
    return gsplat_core


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)
