"""The benchmark's output contract, without a GPU: the reference arm's JSON
line (it runs the reference's CPU code, so it runs here), the kernel count
the GPU arm claims, and the clock sampler's behaviour without a device."""
from __future__ import annotations

import importlib.util
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench():
    spec = importlib.util.spec_from_file_location("bench_under_test",
                                                  os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_reference_arm_line():
    """`--impl reference` prints one JSON line with the metric, the CPU
    baseline it measured and an e2e block with no copies."""
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                          "--workload", "cfg1", "--steps", "1", "--warmup", "3"],
                         check=True, capture_output=True, text=True, timeout=600,
                         cwd=ROOT).stdout
    lines = [ln for ln in out.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unit"] == "Mpix/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["steps"] == 1 and d["warmup"] == 3
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["cores"] >= 1
    assert cb["kind"] in ("reference", "port") and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "Mpix/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}
    # the reference path lists the GPU step's intersections (Metal culling)
    assert d["config"]["isects_per_camera"] == 38_876


def test_kernel_count_matches_launch_list():
    """The GPU arm's gpu_launches claim per config-3 step: 28 kernels, as the
    committed ncu launch list of one step shows."""
    b = _bench()
    passes = b.bin_sort_passes(1, 82, 53)
    assert passes == 5
    assert b.our_kernel_launches(passes, b.bin_count(1, 82, 53), 82 * 53) == 28


def test_clock_sampler_without_device():
    b = _bench()
    c = b.ClockSampler("GPU-none")
    c.start()
    c.begin()
    c.end()
    r = c.stop()
    assert r["sm_mhz"] is None or r["sm_mhz"] > 0
