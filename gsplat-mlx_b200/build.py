"""Build libgsplat_b200.so (the C ABI of include/gsplat_b200.h) in-tree.

nvcc compiles every csrc/*.cu for sm_100a only and links one shared
library next to the Python package (gsplat_core/libgsplat_b200.so), so the
built file travels with the working tree.  No torch, no JIT cache.

    python gsplat-mlx_b200/build.py [--verbose-ptxas] [--force]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
OUT = os.path.join(HERE, "gsplat_core", "libgsplat_b200.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O2", "--expt-relaxed-constexpr",
          "-I" + INCLUDE]
# Files whose float results must round exactly like the reference's CPU code
# (integer keys and radii are derived from them): no FMA contraction.
NO_FMA = {"projection.cu", "intersect.cu", "densify.cu", "export.cu"}


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))


def _compile(src: str, ptxas_verbose: bool) -> tuple[str, str]:
    obj = os.path.join(BUILD, src.replace(".cu", ".o"))
    cmd = [nvcc(), *ARCH, *COMMON, "-c", os.path.join(CSRC, src), "-o", obj]
    cmd.append("-fmad=false" if src in NO_FMA else "-fmad=true")
    if ptxas_verbose:
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def up_to_date() -> bool:
    if not os.path.exists(OUT):
        return False
    t = os.path.getmtime(OUT)
    deps = [os.path.join(CSRC, f) for f in os.listdir(CSRC)] + [
        os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE)] + [os.path.abspath(__file__)]
    return all(os.path.getmtime(d) <= t for d in deps)


def build(force: bool = False, ptxas_verbose: bool = False, quiet: bool = False) -> str:
    if not force and not ptxas_verbose and up_to_date():
        return OUT
    os.makedirs(BUILD, exist_ok=True)
    srcs = sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        results = list(ex.map(lambda s: _compile(s, ptxas_verbose), srcs))
    if ptxas_verbose:
        for s, (_, log) in zip(srcs, results):
            print(f"== {s}\n{log}")
    objs = [o for o, _ in results]
    cmd = [nvcc(), *ARCH, "-shared", "-o", OUT, *objs, "-lcudart_static", "-lrt", "-ldl", "-lpthread"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    if not quiet:
        print(f"built {OUT}")
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose-ptxas", action="store_true")
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args()
    build(force=args.force, ptxas_verbose=args.verbose_ptxas)
    sys.exit(0)
