"""The C ABI library (CPU-only checks; no kernel is launched): it loads,
exports every function include/gsplat_b200.h declares, the ctypes
declarations agree with the header, and host-side helpers behave."""
from __future__ import annotations

import ctypes as ct
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "gsplat_b200.h")


def _declarations():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    decls = {}
    for m in re.finditer(r"\b([A-Za-z_][\w \*]*?)\b(gs_\w+)\s*\(([^;{]*?)\)\s*;", text):
        name, args = m.group(2), m.group(3).strip()
        n = 0 if args in ("", "void") else len([a for a in args.split(",") if a.strip()])
        decls[name] = n
    return decls


def test_header_declares_the_surface():
    d = _declarations()
    for name in ("gs_projection_fwd", "gs_projection_bwd", "gs_quat_scale_to_covar_fwd",
                 "gs_quat_scale_to_covar_bwd", "gs_sh_fwd", "gs_sh_bwd", "gs_isect_tile_count",
                 "gs_isect_scan", "gs_isect_tile_encode", "gs_isect_sort", "gs_isect_offset",
                 "gs_rasterize_fwd", "gs_rasterize_bwd"):
        assert name in d, name


def test_library_exports_every_declared_symbol(gs):
    lib = gs.load()
    for name in _declarations():
        assert hasattr(lib, name), f"{name} not exported"


def test_ctypes_signatures_match_header(gs):
    from gsplat_core._lib import SIGNATURES
    decls = _declarations()
    assert set(SIGNATURES) == set(decls), set(SIGNATURES) ^ set(decls)
    for name, (_, args) in SIGNATURES.items():
        assert len(args) == decls[name], f"{name}: ctypes {len(args)} args, header {decls[name]}"


def test_param_struct_layouts(gs, tmp_path):
    """Every ctypes mirror has the size and field offsets that the C
    compiler gives the header's struct (compiled and run here)."""
    import shutil
    import subprocess
    from gsplat_core import _lib as L
    cc = shutil.which("cc") or shutil.which("gcc")
    if cc is None:
        pytest.skip("no C compiler")
    pairs = {"gs_qs2c_params": L.QS2CParams, "gs_projection_params": L.ProjectionParams,
             "gs_sh_params": L.SHParams, "gs_sh_glue_params": L.SHGlueParams,
             "gs_isect_params": L.IsectParams, "gs_raster_params": L.RasterParams,
             "gs_adam_params": L.AdamParams, "gs_densify_params": L.DensifyParams,
             "gs_densify_mask_params": L.DensifyMaskParams, "gs_spz_params": L.SpzParams}
    lines = []
    for cname, py in pairs.items():
        lines.append(f'printf("{cname} %zu\\n", sizeof({cname}));')
        for f, _ in py._fields_:
            lines.append(f'printf("{cname}.{f} %zu\\n", offsetof({cname}, {f}));')
    src = tmp_path / "layout.c"
    src.write_text("#include <stddef.h>\n#include <stdio.h>\n#include \"gsplat_b200.h\"\n"
                   "int main(void) {\n" + "\n".join(lines) + "\nreturn 0;\n}\n")
    exe = tmp_path / "layout"
    subprocess.run([cc, "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    out = dict(line.split() for line in subprocess.run([str(exe)], check=True, capture_output=True,
                                                       text=True).stdout.splitlines())
    for cname, py in pairs.items():
        assert int(out[cname]) == ct.sizeof(py), cname
        for f, _ in py._fields_:
            assert int(out[f"{cname}.{f}"]) == getattr(py, f).offset, f"{cname}.{f}"


def test_host_helpers(gs):
    lib = gs.load()
    assert lib.gs_version() >= 100
    assert lib.gs_status_string(0) == b"ok"
    assert lib.gs_status_string(5).startswith(b"workspace")
    # floor(log2(x)) + 1 of the reference (gsplat_intersect.cpp:60-65)
    for v, e in [(1, 1), (2, 2), (3, 2), (4, 3), (4346, 13), (8192, 14), (32400, 15)]:
        assert gs.floor_log2_plus_one(v) == e
    assert lib.gs_isect_sort_workspace_size(1000) > 12 * 1000
    assert lib.gs_isect_scan_workspace_size(1 << 20) >= 8 * 256


def test_invalid_arguments_rejected_before_launch(gs):
    """Bad parameters return GS_ERR_INVALID with a message and launch
    nothing (safe without a GPU)."""
    from gsplat_core import _lib as L
    lib = gs.load()
    p = L.IsectParams(0, 10, 16, 4, 4)
    assert lib.gs_isect_tile_count(ct.byref(p), None, None, None, None) == L.GS_ERR_INVALID
    assert b"I * N" in lib.gs_last_error()
    sp = L.SHParams(10, 4, 5, 0)
    assert lib.gs_sh_fwd(ct.byref(sp), None, None, None, None, None) == L.GS_ERR_INVALID
    assert b"degree 0..4" in lib.gs_last_error()
    assert lib.gs_isect_sort(10, 70, None, None, None, None, None, 0, None) == L.GS_ERR_INVALID
    rp = L.RasterParams(1, 1, 3, 16, 16, 64, 1, 1, 0, 0, 0, 0)
    assert lib.gs_rasterize_fwd(ct.byref(rp), *([None] * 12)) == L.GS_ERR_INVALID
    pp = L.ProjectionParams(1, 1, 1, 8, 8, 0.3, 0.01, 1e10, 0.0, 0, 1, 0, 0)
    assert lib.gs_projection_bwd(ct.byref(pp), *([None] * 19)) == L.GS_ERR_INVALID
    assert b"pinhole only" in lib.gs_last_error()


def test_binned_encode_and_densify_validate_before_device_work(gs):
    """Bad arguments of the binned encode and the densify entries come back
    as GS_ERR_INVALID with a message, before any device call (runs on a
    machine without a GPU)."""
    from gsplat_core import _lib as L
    lib = gs.load()
    p = L.IsectParams(1, 10, 16, 4, 4, 0, 0, 0)
    # more bin entries than intersections cannot come from one count
    rc = lib.gs_isect_tile_encode_binned(ct.byref(p), None, None, None, 5, 6, None, None, None,
                                         None, 0, None)
    assert rc == L.GS_ERR_INVALID and b"bin entry" in lib.gs_last_error()
    wide = L.IsectParams(1, 10, 16, 70000, 2, 0, 0, 0)
    rc = lib.gs_isect_tile_encode_binned(ct.byref(wide), None, None, None, 5, 5, None, None, None,
                                         None, 0, None)
    assert rc == L.GS_ERR_INVALID and b"65535" in lib.gs_last_error()
    # SPZ attributes: unknown modes, and SH rest terms with RGB colours
    sp = L.SpzParams(4, 0, 4, 0, 0, 0, 0, 0)
    assert lib.gs_spz_attributes(ct.byref(sp), *([None] * 13)) == L.GS_ERR_INVALID
    sp = L.SpzParams(4, 0, 0, 0, 0, 1, 3, 15)
    assert lib.gs_spz_attributes(ct.byref(sp), *([None] * 13)) == L.GS_ERR_INVALID
    sp = L.SpzParams(4, 0, 0, 0, 0, 0, 0, 0)
    assert lib.gs_spz_attributes(ct.byref(sp), *([None] * 13)) == L.GS_ERR_INVALID
    assert b"missing buffer" in lib.gs_last_error()
    # packed rows: sizes must split into whole images; the encode needs image ids
    assert lib.gs_pack_visible(10, 3, *([None] * 5), 0, *([None] * 7), None, None, 0,
                               None) == L.GS_ERR_INVALID
    assert lib.gs_isect_tile_encode_binned_packed(ct.byref(p), None, None, None, None, 5, 5,
                                                  None, None, None, None, 0, None) == \
        L.GS_ERR_INVALID
    assert b"image_ids" in lib.gs_last_error()
    # the host store of a few totals is bounded and needs both buffers
    assert lib.gs_store_to_host_i64(None, None, 2000, None) == L.GS_ERR_INVALID
    assert lib.gs_store_to_host_i64(None, None, 2, None) == L.GS_ERR_INVALID
    assert lib.gs_store_to_host_i64(None, None, 0, None) == L.GS_OK
    # the tile-culled encode needs the rasterizer's conics and opacities
    rc = lib.gs_isect_tile_encode_binned_culled(ct.byref(p), None, None, None, None, None, 5, 5,
                                                None, None, None, None, None, 0, None)
    assert rc == L.GS_ERR_INVALID and b"conics and opacities" in lib.gs_last_error()
    assert lib.gs_isect_tile_encode_binned_workspace_size(ct.byref(L.IsectParams(0, 10, 16, 4, 4,
                                                                                0, 0, 0)), 5) == 0
    assert lib.gs_isect_tile_count_totals(ct.byref(p), None, None, None, None, None) == \
        L.GS_ERR_INVALID
    dp = L.DensifyParams(0, 10, 8, 8, 1)
    assert lib.gs_densify_accumulate(ct.byref(dp), None, None, None, None, None, None) == \
        L.GS_ERR_INVALID
    mp = L.DensifyMaskParams()
    mp.n = 4
    assert lib.gs_densify_masks(ct.byref(mp), None, None, None, None, None, None, None, None,
                                None, None) == L.GS_ERR_INVALID
    assert b"totals" in lib.gs_last_error()
