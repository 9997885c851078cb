#!/usr/bin/env python
"""Benchmark of the gsplat_core hot path on B200.

A step is one forward + backward pass of the 3DGS training step over the
benchmark scene (gsplat_core.pipeline.TrainingStep): projection, SH colour
glue, tile intersection (count, scan, encode, radix sort, offsets),
rasterize forward and backward, projection backward, SH backward.

Default workload (N=1): benchmark config 3 -- 1M Gaussians, SH degree 3,
one 1297x840 camera.  With --gpus N (torchrun, one rank per GPU) every rank
renders its own camera of the same scene (weak scaling) and the
per-Gaussian gradients are summed with one NCCL all-reduce per step.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line (rank 0).  `value` is Mpix/s over all ranks; ms/step and
intersections sorted/s ride along.  The reference arm times the
reference's own CPU code (eval_cpu compiled from the reference sources,
oracle/_ref) -- or the C restatement when that build is absent -- running
full steps of the same workload on every host thread (oracle/ref_step.py).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "gsplat-mlx_b200"))
sys.path.insert(0, ROOT)

METRIC = "fwd+bwd ms/step and Mpix/s at 1M Gaussians SH3; intersections sorted/s"
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
# measured peer copy per direction per GPU on this pool (NVLink 5; 900 nominal)
LINK_GBS = 770.0
# DRAM bytes (read + write) per launch of each stage's dominant kernel from
# one ncu capture of this benchmark (the committed ncu summaries); None = not
# captured.  Valid for the config-3 workload only.
PROFILED_TRAFFIC = {"rasterize_bwd": 47.1e6, "rasterize_fwd": 19.0e6,
                    "sh_bwd": 120.0e6 + 151.8e6, "projection_bwd": 86.4e6 + 13.7e6}


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return d, "measured"
    except (OSError, ValueError):
        return PEAKS_FALLBACK, "fallback"


WORKLOADS = {
    # name: (description, scaling, cameras_total(world) or None = one per rank)
    "cfg3": ("cfg3: N=1M SH3 Gaussians, 1 camera 1297x840 per GPU, tile 16", "weak"),
    "cfg1": ("cfg1: N=10k SH0 Gaussians (colours as degree-0 SH), 1 camera 256x256 per GPU",
             "weak"),
    "cfg4": ("cfg4: N=3M SH3 Gaussians, 32 cameras 1920x1080 sharded over the GPUs", "strong"),
    "cfg5": ("cfg5: N=6M SH3 Gaussians (log-scales U[-3,-1]), 8 cameras 3840x2160 sharded "
             "over the GPUs", "strong"),
    "cfg2": ("cfg2: 2D image fitting, N=100k, 512x512, L2 loss, MLX Adam lr 1e-2; one step = "
             "render + loss + backward + Adam, loss read on the host every step", "replicas"),
}


def _rotated(sc, rank, world):
    """The scene seen from its first camera rotated by 2 pi rank / world
    about the vertical axis through the origin."""
    from gsplat_core import synthetic as S
    if rank == 0:
        return sc.viewmats[:1]
    R, t = sc.viewmats[0, :3, :3], sc.viewmats[0, :3, 3]
    p0 = -R.T @ t
    th = 2.0 * np.pi * rank / max(world, 1)
    rot = np.array([[np.cos(th), 0, np.sin(th)], [0, 1, 0], [-np.sin(th), 0, np.cos(th)]])
    return S.look_at(rot @ p0)[None].astype(np.float32)


def scene_for(rank, world, seed, workload="cfg3"):
    """The workload's scene with every camera of the job in viewmats / Ks:
    weak workloads give rank r its own camera (the first camera rotated),
    strong ones keep the config's cameras."""
    from gsplat_core import synthetic as S
    if workload == "cfg3":
        sc = S.config3(seed=seed)
    elif workload == "cfg1":
        sc = S.config1(seed=seed)
        # colours passed directly (render_random_3dgs_png.py) expressed as the
        # degree-0 SH coefficient that the clamp glue maps back to them
        sc.coeffs = ((sc.colors - 0.5) / 0.28209479177387814)[:, None, :].astype(np.float32)
        sc.sh_degree = 0
    elif workload == "cfg2":
        sc = S.config2(seed=seed)
        sc.coeffs = ((sc.colors - 0.5) / 0.28209479177387814)[:, None, :].astype(np.float32)
        sc.sh_degree = 0
        return sc
    elif workload == "cfg4":
        return S.config4(seed=seed)
    elif workload == "cfg5":
        return S.config5(seed=seed)
    else:
        raise ValueError(workload)
    sc.viewmats = np.concatenate([_rotated(sc, r, world) for r in range(world)])
    sc.Ks = np.repeat(sc.Ks[:1], world, 0)
    return sc


# ------------------------------------------------------------------ clocks

class ClockSampler:
    """Clocks and throttle reasons while the timed region runs: nvidia-smi
    every 200 ms, and NVML (read-only queries) every 5 ms from a thread, so
    that a timed region shorter than nvidia-smi's interval is sampled too."""

    # NVML clock event reason bits
    NVML_REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40,
                    "sw_thermal_slowdown": 0x20, "sw_power_cap": 0x4}

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id):
        self.gpu = gpu_id
        self.proc = None
        self.lines = []
        self.nvml = []  # (sm MHz, max sm MHz, reason bits), inside begin() .. end()
        self._stop = threading.Event()
        self._active = threading.Event()
        self.nt = None
        self._h = None
        self._smax = 0.0

    def begin(self):
        """The timed region starts: NVML samples are kept from here on (one
        is taken at once, one more at end())."""
        self._sample()
        self._active.set()

    def end(self):
        self._active.clear()
        self._sample()

    def _sample(self):
        if self._h is None:
            return
        try:
            import pynvml
            sm = pynvml.nvmlDeviceGetClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            bits = pynvml.nvmlDeviceGetCurrentClocksEventReasons(self._h)
            self.nvml.append((float(sm), self._smax, int(bits)))
        except Exception:
            pass

    def _nvml_open(self):
        self._h = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self._h = pynvml.nvmlDeviceGetHandleByUUID(self.gpu)
            self._smax = float(pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM))
        except Exception:  # no NVML binding or library: nvidia-smi alone
            self._h = None

    def _nvml_loop(self):
        while not self._stop.wait(0.005):
            if self._active.is_set():
                self._sample()

    def start(self):
        self._nvml_open()
        if self._h is not None:
            self.nt = threading.Thread(target=self._nvml_loop, daemon=True)
            self.nt.start()
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        self._stop.set()
        if self.nt is not None:
            self.nt.join(timeout=5)
        if self._h is not None:
            try:
                import pynvml
                pynvml.nvmlShutdown()
            except Exception:
                pass
        sm, smax, reasons = [], [], set()
        for c, cm, bits in self.nvml:
            sm.append(c)
            smax.append(cm)
            reasons.update(nm for nm, b in self.NVML_REASONS.items() if bits & b)
        if self.proc is None:
            if not sm:
                return {"sm_mhz": None, "sm_max_mhz": None,
                        "reasons": ["nvidia-smi unavailable"]}
        else:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": float(np.median(sm)) if sm else None,
                "sm_max_mhz": float(max(smax)) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm),
                "nvml_samples": len(self.nvml)}


# ------------------------------------------------------------------ helpers

def algorithmic_bytes(stage, N, C, visible, m, pixels, K, slots, kept=None):
    """Bytes each stage must move at minimum (the roofline convention): what
    it reads once and writes once, not what an implementation's intermediate
    passes move.  N Gaussians seen by C cameras (C N elements); ``visible``:
    Gaussians some camera sees, whose coefficient rows the fused SH kernels
    read (and write) once for all cameras; ``slots``: tile offsets written;
    ``kept``: the intersections left after the encode's tile culling (the
    lists the rasterizers walk), else m."""
    mk = m if kept is None else kept
    e = N * C
    return {
        # means/quats/scales in once (40 B), 2D outputs out (36 B) per element
        "projection_fwd": N * 40 + e * 36,
        # means in, campos per camera, colours out per element; the
        # coefficient row of every visible Gaussian once
        "sh_fwd": N * 12 + C * 16 + e * 12 + visible * K * 12,
        # rects from means2d/radii, counts out, their total
        "isect_count": e * (16 + 4),
        # means2d, radii, depths in; sorted keys + flatten ids and the tile
        # offsets out (the binned encode writes the offsets itself)
        "isect_encode_sort": e * (8 + 8 + 4) + mk * 12 + slots * 4,
        "isect_offset": m * 8,
        # opacity in, its two sigma bounds out
        "sigma_bounds": N * (4 + 8),
        # tile offsets (forward) or the forward's tile costs (backward) in,
        # the schedule out
        "tile_order": slots * 8,
        "tile_order_bwd": slots * 8,
        # per intersection: flatten id + Gaussian record; per pixel: outputs
        "rasterize_fwd": mk * 40 + pixels * 20,
        "rasterize_bwd": mk * (40 + 36) + pixels * 20,
        # per element: radii, conics, cotangents; per Gaussian: parameters in,
        # gradients out
        "projection_bwd": e * (8 + 12 + 8 + 4 + 12) + N * (40 + 40),
        # means in and v_means out per Gaussian, v_colours in per element,
        # coefficient rows of visible Gaussians in, every v_coeffs row out
        "sh_bwd": N * (12 + 12) + e * 12 + visible * K * 12 + N * K * 12,
    }[stage]


# Warp instructions per launch of the rasterizers at config 3 (one pass of
# `ncu --metrics gpu__time_duration.sum,smsp__inst_executed.sum`,
# the committed launch-list summary): their roofline is the SMs' instruction issue,
# 148 SMs x 4 schedulers x the sampled SM clock, not HBM.
PROFILED_INSTS = {"rasterize_bwd": 356_746_241 + 9_720,  # + its tile-order kernel
                  # the forward kernel, its tile-order kernel and the exact
                  # fix-up kernel
                  "rasterize_fwd": 199_708_576 + 9_720 + 6_687_814}


def bin_count(cameras, tw, th):
    """4x4-tile bins of the binned encode."""
    return cameras * -(-tw // 4) * -(-th // 4)


def bin_sort_passes(cameras, tw, th):
    """Radix passes of the binned encode's entry sort: 31 depth bits (the
    training step's depths are positive) plus the bits of the bin ids."""
    return (31 + (bin_count(cameras, tw, th) - 1).bit_length() + 7) // 8


def our_kernel_launches(entry_passes, bins, slots, tile_cull=False):
    # projection fwd 1, glue fwd 1, count (+ totals) 1; binned encode: bin
    # counts 1, their scan 1, entry emit 1, digit histogram 1, entry passes,
    # bin starts + tile masks 1, item counts per bin 1 and their scan, item
    # count phase 1, slot counts 1 and their scan, (tile culling: the offsets'
    # gap 1), item write phase 1 (a scan is one launch up to 16384 values,
    # else 3); rasterize fwd 1, rasterize bwd 1, projection bwd 1, glue bwd 1
    scan = lambda n: 1 if n <= 16384 else 3  # noqa: E731
    binned = (3 + 1 + entry_passes + 1 + 1 + scan(bins) + 1 + 1 + scan(slots) + int(tile_cull)
              + 1)
    # + the sigma bounds of the opacities 1, the totals' store to pinned host
    # memory 1, the rasterizers' tile orders 2, the forward's fix-up pass of
    # undecided pixels 1
    return 1 + 1 + 1 + 1 + binned + 1 + 1 + 1 + 1 + 1 + 2 + 1


# ------------------------------------------------------------------ CPU arms

def cpu_steps(checker, sc, vrc, vra, steps, warmup):
    """The reference's CPU step of one camera, timed in full on every host
    thread (oracle.ref_step: the reference's own eval_cpu code per Gaussian
    chunk / tile set, the Metal culling applied, the same intersections as
    the GPU step).  Returns (seconds per step, intersections, seconds of the
    intersect pipeline per step, threads)."""
    from oracle.ref_step import ParallelReferenceStep
    st = ParallelReferenceStep(checker, sc, vrc, vra)
    try:
        for _ in range(warmup):
            st.run()
        secs, isect = [], []
        m = 0
        for _ in range(steps):
            t, m, ti = st.run()
            secs.append(t)
            isect.append(ti)
    finally:
        st.close()
    return float(np.mean(secs)), m, float(np.mean(isect)), st.T


def composited_pairs(step):
    """Pixel x Gaussian pairs the backward evaluates: per pixel, the
    intersections of its tile from the first up to its last composited one
    (sum over this rank's images)."""
    import torch
    li = step.last_ids.long()
    offs = step.tile_offsets.long()
    ty = torch.arange(step.H, device=li.device) // step.ts
    tx = torch.arange(step.W, device=li.device) // step.ts
    start = offs[:, ty][:, :, tx]
    return int((li - start + 1).clamp(min=0).sum().item())


def first_camera(sc):
    """The scene restricted to its first camera (CPU baseline sample)."""
    import dataclasses
    return dataclasses.replace(sc, viewmats=sc.viewmats[:1], Ks=sc.Ks[:1])


def make_checker():
    from oracle.oracle import Oracle, Reference
    if Reference.available():
        return Reference(), "reference"
    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), "oracle"], check=False)
    return Oracle(), "port"


def run_reference_arm(args):
    """The reference's CPU path on the same workload: each step is one full
    camera step (every Gaussian, every tile, forward and backward), timed
    wall-clock on all host threads; multi-camera workloads time one camera
    per step and scale by the camera count (stated in `sample`).  Under
    torchrun only rank 0 runs."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    from gsplat_core import synthetic as S
    checker, kind = make_checker()
    full_sc = scene_for(0, 1, args.seed, args.workload)
    cams = full_sc.cameras
    sc = first_camera(full_sc)
    vrc, vra = S.cotangents(args.seed, 1, sc.height, sc.width)
    sec, m, t_isect, threads = cpu_steps(checker, sc, vrc, vra, args.steps, args.warmup)
    ms = 1e3 * sec * cams
    pixels = sc.width * sc.height * cams
    value = pixels / (ms / 1e3) / 1e6
    sample = (f"{args.workload}: every step one full camera step timed wall-clock "
              f"(projection, SH, intersect on all {sc.n} Gaussians, rasterize fwd+bwd on all "
              f"{sc.tile_width * sc.tile_height} tiles, SH and projection backward) on "
              f"{threads} host threads" +
              (f"; x{cams} cameras (one camera per step, scaled)" if cams > 1 else ""))
    out = {"impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "Mpix/s",
           "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
           "ms_per_step": round(ms, 3), "higher_is_better": True,
           "scaling": WORKLOADS[args.workload][1], "vs_baseline": None, "dtype": "f32",
           "data": f"synthetic (seeded, benchmark {args.workload} shapes)",
           "config": {"workload": WORKLOADS[args.workload][0], "cameras": cams,
                      "gaussians": sc.n, "isects_per_camera": m},
           "intersections_sorted_per_s": round(m / t_isect, 1),
           "cpu_baseline": {"value": round(value, 4), "unit": "Mpix/s", "cores": threads,
                            "kind": kind, "sample": sample},
           "e2e": {"value": round(value, 4), "unit": "Mpix/s", "h2d_bytes_per_step": 0,
                   "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)
    return 0


# ------------------------------------------------------------------ GPU arm

def run_fit(args):
    """benchmark config 2: the image-fitting trainer's step on device
    (gsplat_core.fitting), the loss read back every step as the trainer
    does; with N GPUs every rank fits its own copy (replicas)."""
    import torch
    import torch.distributed as dist
    from gsplat_core import fitting, synthetic as S
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    sc = S.config2(seed=args.seed)
    target = S.fitting_target(args.seed, sc.width, sc.height)
    logit = lambda x: np.log(np.clip(x, 1e-5, 1 - 1e-5) / (1 - np.clip(x, 1e-5, 1 - 1e-5)))  # noqa
    fit = fitting.ImageFitStep(sc.means, sc.quats, np.log(sc.scales), logit(sc.colors),
                               logit(sc.opacities), sc.viewmats[0], sc.Ks[0], target, sc.width,
                               sc.height, device=dev)
    losses = [float(fit.run().item()) for _ in range(args.warmup)]
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = ClockSampler("GPU-" + str(torch.cuda.get_device_properties(dev).uuid))
    clocks.start()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    clocks.begin()
    t0.record()
    for _ in range(args.steps):
        losses.append(float(fit.run().item()))   # the trainer's per-step loss read
    t1.record()
    torch.cuda.synchronize()
    clocks.end()
    clk = clocks.stop()
    t = torch.tensor([t0.elapsed_time(t1)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item()) / args.steps
    if rank == 0:
        out = {"metric": METRIC, "value": round(sc.width * sc.height * world / ms / 1e3, 3),
               "unit": "Mpix/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
               "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
               "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded, benchmark cfg2)",
               "config": {"workload": WORKLOADS["cfg2"][0], "gaussians": sc.n,
                          "isects_last_step": fit.step.m,
                          "loss_first": losses[0], "loss_last": losses[-1],
                          "steps_run": len(losses)},
               "gpu_launches": None, "clocks": clk}
        print(json.dumps(out), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_ours(args):
    import torch
    import torch.distributed as dist
    from gsplat_core import synthetic as S
    from gsplat_core.sharded import ShardedTrainingStep, exchange_bytes

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    desc, scaling = WORKLOADS[args.workload]
    sc = scene_for(rank, world, args.seed, args.workload)
    C_total = sc.cameras
    from gsplat_core.sharded import camera_shard
    c0, c1 = camera_shard(C_total, world, rank)
    vrc_np, vra_np = S.cotangents(args.seed + rank, c1 - c0, sc.height, sc.width)
    # every rank holds the poses of all cameras (the SH exchange recomputes
    # the colour basis of remote cameras)
    host = {"means": sc.means, "quats": sc.quats, "scales": sc.scales,
            "opacities": sc.opacities, "coeffs": sc.coeffs, "viewmats": sc.viewmats,
            "Ks": sc.Ks, "v_render_colors": vrc_np, "v_render_alphas": vra_np}
    order = list(host)
    d = {k: torch.from_numpy(np.ascontiguousarray(v)).to(dev) for k, v in host.items()}
    pinned = {k: torch.from_numpy(np.ascontiguousarray(v)).pin_memory() for k, v in host.items()}
    sharded = ShardedTrainingStep(sc.n, sc.sh_degree, sc.coeffs.shape[1], C_total, sc.width,
                                  sc.height, exchange=args.exchange, device=dev,
                                  tile_cull=args.tile_cull)
    step = sharded.step
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)

    def one(inp):
        flat, m = sharded.run(*[inp[k] for k in order])
        if world > 1:
            step._mark("exchange")
        return m

    for _ in range(args.warmup):
        one(d)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()

    # ---- timed region: K steps, device-resident inputs, L2 flushed between
    try:
        gpu_id = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:  # older torch: fall back to the ordinal
        gpu_id = str(local)
    clocks = ClockSampler(gpu_id)
    clocks.start()
    time.sleep(0.3)
    step.events = []
    stage_ms = {}
    step_ms = []
    m = 0
    clocks.begin()
    for _ in range(args.steps):
        flush.fill_(1.0)
        s_ev = torch.cuda.Event(enable_timing=True)
        e_ev = torch.cuda.Event(enable_timing=True)
        step.events = []
        s_ev.record()
        m = one(d)
        e_ev.record()
        torch.cuda.synchronize()
        step_ms.append(s_ev.elapsed_time(e_ev))
        evs = step.events
        this = {}
        for (n0, a), (n1, b) in zip(evs[:-1], evs[1:]):
            if n1 != "start":
                this[n1] = this.get(n1, 0.0) + a.elapsed_time(b)
        # stages on the side stream, beside the intersect pipeline
        for n1, a, b in getattr(step, "side_spans", []):
            this[n1] = this.get(n1, 0.0) + a.elapsed_time(b)
        for k, v in this.items():
            stage_ms.setdefault(k, []).append(v)
    step.events = None
    clocks.end()
    clk = clocks.stop()
    local_ms = float(np.sum(step_ms))
    t = torch.tensor([local_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms = float(t.item())
    ms_step = total_ms / args.steps
    pixels = sc.width * sc.height * C_total       # the whole job's pixels per step
    value = pixels * args.steps / (total_ms / 1e3) / 1e6

    # ---- e2e: the same step driven from pinned host buffers.  Every step
    # uploads all of its inputs (Gaussian parameters, cameras, image
    # cotangents) and downloads its whole flat gradient.  Uploads and
    # downloads run on their own streams, double-buffered, so that step k+1's
    # upload and step k's download overlap step k's kernels (PCIe is full
    # duplex).  Timed on the device from the first upload to the last
    # download; the inputs (253 MB) exceed L2, so no flush is added.
    h2d_s = torch.cuda.Stream(device=dev)
    d2h_s = torch.cuda.Stream(device=dev)
    comp = torch.cuda.current_stream(dev)
    bufs = [{k: torch.empty_like(d[k]) for k in order} for _ in range(2)]
    stage = [torch.empty_like(step.grad_flat) for _ in range(2)]
    grad_host = [torch.empty(step.grad_flat.shape, dtype=torch.float32).pin_memory()
                 for _ in range(2)]
    h2d_done = [torch.cuda.Event() for _ in range(2)]
    comp_done = [torch.cuda.Event() for _ in range(2)]
    d2h_done = [torch.cuda.Event() for _ in range(2)]
    h2d = sum(v.numel() * v.element_size() for v in pinned.values())
    d2h = grad_host[0].numel() * 4

    def upload(k):
        b = k % 2
        if k >= 2:
            h2d_s.wait_event(comp_done[b])      # step k-2 has consumed buffer b
        with torch.cuda.stream(h2d_s):
            for name in order:
                bufs[b][name].copy_(pinned[name], non_blocking=True)
        h2d_done[b].record(h2d_s)

    def run_e2e(n_steps):
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(h2d_s)
        upload(0)
        for k in range(n_steps):
            b = k % 2
            if k + 1 < n_steps:
                upload(k + 1)
            comp.wait_event(h2d_done[b])
            if k >= 2:
                comp.wait_event(d2h_done[b])    # staging buffer b downloaded
            one(bufs[b])
            # staged by a kernel (an elementwise copy), not a memcpy that a
            # copy engine busy with the previous download would hold back
            torch.mul(step.grad_flat, 1.0, out=stage[b])
            comp_done[b].record(comp)
            d2h_s.wait_event(comp_done[b])
            with torch.cuda.stream(d2h_s):
                grad_host[b].copy_(stage[b], non_blocking=True)
            d2h_done[b].record(d2h_s)
        t1.record(d2h_s)
        torch.cuda.synchronize()
        return t0.elapsed_time(t1)

    run_e2e(args.warmup)
    t = torch.tensor([run_e2e(args.steps)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_value = pixels * args.steps / (float(t.item()) / 1e3) / 1e6

    if rank == 0:
        peaks, peak_kind = load_peaks()
        hbm = float(peaks.get("hbm_gbs", PEAKS_FALLBACK["hbm_gbs"]))
        vis_el = (step.radii[..., 0] > 0) & (step.radii[..., 1] > 0)
        visible = int(vis_el.sum().item())
        visible_any = int(vis_el.any(dim=0).sum().item())
        K = sc.coeffs.shape[1]
        passes = bin_sort_passes(sharded.C, sc.tile_width, sc.tile_height)
        slots = sharded.C * sc.tile_width * sc.tile_height
        avg = {k: float(np.mean(v)) for k, v in stage_ms.items()}
        top = max((k for k in avg if k != "exchange"), key=avg.get)
        # this rank's units: N Gaussians, C cameras, pixels
        pix_local = sc.width * sc.height * sharded.C
        kept = step.kept_isects() if step.bands == 1 else None
        sm_mhz = clk.get("sm_mhz") or clk.get("sm_max_mhz") or 1965.0
        issue_peak = 148 * 4 * sm_mhz * 1e6 / 1e9  # G warp instructions / s
        bytes_of = lambda k: algorithmic_bytes(k, sc.n, sharded.C, visible_any, m,  # noqa: E731
                                               pix_local, K, slots, kept)
        stages = {}
        for k, v in avg.items():
            if k == "exchange":
                # NCCL exchange (+ the SH glue backward over all cameras in
                # gather mode): bytes each rank sends, against the link
                b = exchange_bytes(sharded.exchange, sc.n, K, step.C, world)
                stages[k] = {"ms": round(v, 4), "mode": sharded.exchange,
                             "GBps_sent": round(b / (v / 1e3) / 1e9, 1),
                             "frac_link": round(b / (v / 1e3) / 1e9 / LINK_GBS, 4)}
                continue
            b = bytes_of(k)
            stages[k] = {"ms": round(v, 4), "GBps": round(b / (v / 1e3) / 1e9, 1),
                         "frac_hbm": round(b / (v / 1e3) / 1e9 / hbm, 4)}
            if k in PROFILED_INSTS and args.workload == "cfg3" and sharded.C == 1:
                ginst = PROFILED_INSTS[k] / (v / 1e3) / 1e9
                stages[k]["Ginst_per_s"] = round(ginst, 1)
                stages[k]["frac_issue"] = round(ginst / issue_peak, 4)
        if top in PROFILED_INSTS and args.workload == "cfg3" and sharded.C == 1:
            ginst = PROFILED_INSTS[top] / (avg[top] / 1e3) / 1e9
            roofline = {"kernel": top, "bound": "issue", "achieved": round(ginst, 1),
                        "peak": round(issue_peak, 1), "unit": "G warp-instructions/s",
                        "frac": round(ginst / issue_peak, 4),
                        "peak_source": "148 SMs x 4 schedulers x median sampled SM clock",
                        "warp_instructions": int(PROFILED_INSTS[top]),
                        "traffic": PROFILED_TRAFFIC.get(top),
                        "algorithmic_bytes": int(bytes_of(top)),
                        "frac_hbm": round(bytes_of(top) / (avg[top] / 1e3) / 1e9 / hbm, 4)}
        else:
            achieved = bytes_of(top) / (avg[top] / 1e3) / 1e9
            roofline = {"kernel": top, "bound": "hbm", "achieved": round(achieved, 1),
                        "peak": hbm, "unit": "GB/s", "frac": round(achieved / hbm, 4),
                        "peak_source": peak_kind, "traffic": PROFILED_TRAFFIC.get(top),
                        "algorithmic_bytes": int(bytes_of(top))}
        # the step's roofline: the sum over its serial stages of each one's
        # lower bound (algorithmic bytes at the HBM peak; for the rasterizers
        # at config 3 the larger of that and their warp instructions at the
        # issue peak; the exchange's bytes at the link rate) over the step time
        t_min = 0.0
        for k in avg:
            if k == "sigma_bounds":  # on a side stream, beside the encode
                continue
            if k == "exchange":
                t_min += exchange_bytes(sharded.exchange, sc.n, K, step.C, world) / (
                    LINK_GBS * 1e9) * 1e3
                continue
            t = bytes_of(k) / (hbm * 1e9) * 1e3
            if k in PROFILED_INSTS and args.workload == "cfg3" and sharded.C == 1:
                t = max(t, PROFILED_INSTS[k] / (issue_peak * 1e9) * 1e3)
            t_min += t
        step_roofline = {"t_min_ms": round(t_min, 4), "frac": round(t_min / ms_step, 4),
                         "how": "sum over the serial stages of max(algorithmic bytes / HBM "
                                "peak, warp instructions / issue peak), exchange bytes / link"}
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            checker, kind = make_checker()
            sc0 = first_camera(sc)
            sec, _, _, threads = cpu_steps(checker, sc0, vrc_np[:1], vra_np[:1],
                                           args.cpu_steps, 1)
            cpu = {"value": round(sc0.width * sc0.height / sec / 1e6, 4), "unit": "Mpix/s",
                   "cores": threads, "kind": kind,
                   "sample": (f"{args.cpu_steps} full steps of one camera of the "
                              f"{args.workload} step (every tile, forward and backward) after "
                              f"one warm-up step, wall-clock on {threads} host threads; the "
                              f"per-camera rate stands for all {C_total} cameras")}
        out = {
            "metric": METRIC, "value": round(value, 3), "unit": "Mpix/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
            "higher_is_better": True, "scaling": scaling, "vs_baseline": None, "dtype": "f32",
            "data": f"synthetic (seeded, benchmark {args.workload} distributions)",
            "config": {"workload": desc, "cameras": C_total,
                       "gaussians": sc.n, "visible": visible, "visible_any": visible_any,
                       "isects": m,
                       # after the encode's opacity-aware tile culling
                       "isects_kept": kept, "tile_cull": step.tile_cull,
                       # (per band when the step renders bands of tile rows)
                       "bwd_pixel_gaussian_pairs": (composited_pairs(step) if step.bands == 1
                                                    else None),
                       "bands": step.bands,
                       "parallelism": f"camera-sharded dp{world}" if world > 1 else "single",
                       "exchange": sharded.exchange if world > 1 else None,
                       "l2": "flushed (256 MB write) between timed steps"},
            # M / (encode + sort) time of this rank's step
            "intersections_sorted_per_s": round(m / (avg["isect_encode_sort"] / 1e3), 1),
            "stages_ms": stages,
            "roofline": roofline,
            "step_roofline": step_roofline,
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_value, 3), "unit": "Mpix/s", "h2d_bytes_per_step": int(h2d),
                    "d2h_bytes_per_step": int(d2h),
                    "how": "all inputs uploaded and the flat gradient downloaded every step "
                           "from pinned host memory; copies double-buffered on their own "
                           "streams, overlapping the neighbouring steps' kernels"},
            "gpu_launches": our_kernel_launches(
                passes, bin_count(sharded.C, sc.tile_width, sc.tile_height), slots,
                step.tile_cull) * args.steps,
            "clocks": clk,
        }
        print(json.dumps(out), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--cpu-steps", type=int, default=3,
                    help="full reference steps timed for the cpu_baseline field")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="cfg3",
                    help="benchmark config (cfg3 is the headline; the others fill the "
                         "per-config records)")
    ap.add_argument("--exchange", choices=["auto", "allreduce", "gather", "shard"], default="auto",
                    help="gradient exchange of the camera-sharded step (N > 1)")
    ap.add_argument("--tile-cull", action="store_true",
                    help="opacity-aware tile culling in the encode (the renders are the "
                         "same either way; the reference lists every pair of the rects)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference_arm(args)
    if args.workload == "cfg2":
        return run_fit(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
