"""The C++ eval_gpu adapter (gsplat-mlx_b200/adapter/) against the
reference's Primitive classes, without a GPU: it compiles against the
reference's headers, and the device-mode build of the reference's
front-ends (oracle/_ref/libgsplat_ref_cuda.so, used by the GPU test of the
adapter) takes every eval_gpu from the adapter, none from the reference's
throwing fallback (a single global definition of each)."""
from __future__ import annotations

import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ADAPTER = os.path.join(ROOT, "gsplat-mlx_b200", "adapter")
CUDA_SO = os.path.join(ROOT, "oracle", "_ref", "libgsplat_ref_cuda.so")

PRIMITIVES = [
    "GSPlatQuatScaleToCovarPreci", "GSPlatQuatScaleToCovarPreciBackward",
    "GSPlatProjectionEWA3DGSFused", "GSPlatProjectionEWA3DGSFusedBackward",
    "GSPlatSphericalHarmonics", "GSPlatSphericalHarmonicsBackward",
    "GSPlatIntersectTileCount", "GSPlatIntersectTileEncode", "GSPlatIntersectOffset",
    "GSPlatRasterizeToPixels3DGS", "GSPlatRasterizeToPixels3DGSBackward",
]


def _eval_gpu_symbols(path):
    out = subprocess.run(["nm", "-C", "--defined-only", path], check=True,
                         capture_output=True, text=True).stdout
    syms = {}
    for line in out.splitlines():
        parts = line.split(None, 2)
        if len(parts) == 3 and "::eval_gpu(" in parts[2] and "[clone" not in parts[2]:
            cls = parts[2].split("::eval_gpu(")[0].split("::")[-1]
            syms.setdefault(cls, set()).add(parts[1])
    return syms


def test_adapter_defines_every_eval_gpu():
    if not os.path.exists(CUDA_SO):
        pytest.skip("device-mode reference build absent (make -C oracle ref_cuda)")
    syms = _eval_gpu_symbols(CUDA_SO)
    for cls in PRIMITIVES + ["IntersectSort"]:
        assert syms.get(cls) == {"T"}, (cls, syms.get(cls))
    # one definition each: the reference's own (throwing) ones were weak and
    # were dropped by the link (their message strings stay in the data)


def test_adapter_compiles_against_reference_headers(tmp_path):
    ref = os.environ.get("GSPLAT_REF_DIR", "")
    if not ref or not os.path.isdir(os.path.join(ref, "gsplat_core")):
        pytest.skip("GSPLAT_REF_DIR (the reference checkout) not set")
    cuda_inc = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "include")
    obj = tmp_path / "adapter.o"
    subprocess.run(["g++", "-std=c++20", "-O1", "-fPIC", "-Wall", "-Wextra", "-Werror",
                    "-Wno-unused-parameter", f"-I{cuda_inc}",
                    "-I" + os.path.join(ROOT, "oracle", "mlx_shim"), f"-I{ref}",
                    "-I" + os.path.join(ROOT, "include"), f"-I{ADAPTER}", "-c",
                    os.path.join(ADAPTER, "gsplat_b200_eval_gpu.cpp"), "-o", str(obj)],
                   check=True)
    syms = _eval_gpu_symbols(str(obj))
    assert set(PRIMITIVES) <= set(syms)
