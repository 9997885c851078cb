"""Camera-sharded multi-view training step, one process per GPU.

Every (camera, Gaussian) pair, tile and pixel of the hot path is
independent; the only coupling between cameras is the per-Gaussian gradient
sum that the reference's projection backward forms by looping over the
cameras (metal/gsplat_projection.metal:488-545) and that MLX autograd forms
over the trainers' camera loop.  So each rank holds the full Gaussian set,
renders its own contiguous slice of the cameras with ``TrainingStep``, and
the ranks exchange gradients once per step.  Three exchanges give the same
sums (up to fp32 summation order):

* ``"allreduce"`` -- every rank runs the whole backward for its cameras and
  one all-reduce(sum) runs over the flat gradient buffer
  ``[v_means | v_quats | v_scales | v_opacities | v_coeffs]`` (4 (11 + 3K)
  bytes per Gaussian: 236 B at SH degree 3).
* ``"gather"`` -- the SH gradient is a sum over cameras of the colour
  cotangent times a basis that any rank can recompute from the replicated
  means, coefficients and camera poses.  Ranks all-gather the colour
  cotangents ``v_colors`` of their cameras (12 B per Gaussian per camera)
  and all-reduce only the projection part ``[v_means | v_quats | v_scales |
  v_opacities]`` (44 B per Gaussian); each rank then runs the SH glue
  backward over all cameras, which writes the full v_coeffs and adds the
  SH part of v_means.

* ``"shard"`` -- the SH glue backward is split by Gaussian instead of
  replicated: rank q owns the Gaussians [q N/R, (q+1) N/R).  One all-to-all
  per local camera moves each slice of the colour cotangents to its owner
  (started as soon as the rasterizer backward is queued, so it overlaps the
  projection backward); a reduce-scatter sums the projection part per slice;
  each rank runs the SH glue backward for its slice over every camera
  (adding the SH part of v_means into its reduced slice) and one all-gather
  assembles the full gradient on every rank.  Per rank: (R-1)/R (12 C_local
  + 4 (11 + 3K)) N bytes and 1/R of the SH backward, whatever R.  Needs N
  divisible by R.

``"auto"`` picks the exchange that sends the fewest bytes per rank (ring
estimates in ``exchange_bytes``; ties to the one with fewer collective
steps): gather with one camera per rank (config 3's weak scaling), shard
with many cameras per rank and N divisible by R.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def camera_shard(cameras, world, rank):
    """Contiguous, balanced camera slice [start, stop) of ``rank``; the
    first ``cameras % world`` ranks take one camera more."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    base, extra = divmod(int(cameras), int(world))
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def exchange_bytes(mode, n, K, cameras_per_rank, world):
    """Bytes each rank sends per step for an exchange (ring algorithms:
    all-reduce 2 (w-1)/w S, all-gather (w-1) S_rank)."""
    if world <= 1:
        return 0.0
    ring = 2.0 * (world - 1) / world
    if mode == "allreduce":
        return ring * 4.0 * (11 + 3 * K) * n
    if mode == "gather":
        return ring * 44.0 * n + (world - 1) * 12.0 * n * cameras_per_rank
    if mode == "shard":
        part = (world - 1) / world
        return part * (12.0 * cameras_per_rank + 4.0 * (11 + 3 * K)) * n + part * 44.0 * n
    raise ValueError(f"unknown exchange {mode!r}")


def choose_exchange(n, K, cameras_per_rank, world):
    """The exchange that sends the fewest bytes per rank; ties go to the one
    with fewer collective steps (allreduce, then gather, then shard).  The
    shard exchange needs SH coefficients (K > 1) and equal Gaussian slices.
    With one camera per rank the gather exchange sends the least (two
    GPUs, config 3: gather 1.40 ms/step against shard 1.68 ms)."""
    if world <= 1:
        return "allreduce"
    modes = ["allreduce", "gather"] + (["shard"] if K > 1 and n % world == 0 else [])
    return min(modes, key=lambda m: exchange_bytes(m, n, K, cameras_per_rank, world))


# [v_means | v_quats | v_scales | v_opacities] of the flat gradient buffer:
# (offset, width) in units of N floats; v_coeffs follows at 11 N.
PROJ_FIELDS = ((0, 3), (3, 4), (7, 3), (10, 1))


class _Works:
    def __init__(self, works):
        self.works = [w for w in works if w is not None]

    def wait(self):
        for w in self.works:
            w.wait()


def _coalesced(fn, pairs, group, device):
    """Asynchronous collectives ``fn(out, inp)`` over (out, inp) pairs: one
    NCCL group launch (coalescing manager) with NCCL, separate ops with
    gloo.  Returns a handle with wait()."""
    if dist.get_backend(group) == "nccl":
        with dist.distributed_c10d._coalescing_manager(group=group, device=device,
                                                       async_ops=True) as cm:
            for out, inp in pairs:
                fn(out, inp, group=group)
        return cm
    return _Works([fn(out, inp, group=group, async_op=True) for out, inp in pairs])


def start_shard_all_to_all(recv, v_colors_local, group):
    """Moves each Gaussian slice of this rank's colour cotangents
    [C_local, N, 3] to the slice's owner: recv [C_local * R, N / R, 3]
    receives, for local camera j of rank g, row j R + g (the order
    camera_groups = R of the SH glue backward reads)."""
    R = dist.get_world_size(group)
    C_local = v_colors_local.shape[0]
    works = []
    for j in range(C_local):
        works.append(dist.all_to_all_single(recv[j * R:(j + 1) * R].reshape(-1),
                                            v_colors_local[j].reshape(-1), group=group,
                                            async_op=True))
    return _Works(works)


def shard_exchange(grad_flat, n, K, reduced, coeff_slice, sh_slice_backward, moving, group=None,
                   device=None):
    """The "shard" exchange after this rank's projection backward:
    ``grad_flat`` holds this rank's projection part for all N Gaussians;
    ``moving`` is the handle of start_shard_all_to_all.  ``reduced``: the
    four per-slice field buffers ([d N / R] each, see PROJ_FIELDS);
    ``coeff_slice`` [N / R, K, 3].  ``sh_slice_backward()`` runs the SH
    glue backward of this rank's slice over every camera, writing
    coeff_slice and adding the SH part of v_means into reduced[0].
    Afterwards every rank holds the full summed gradient in grad_flat."""
    summing = _coalesced(dist.reduce_scatter_tensor,
                         [(reduced[i], grad_flat[o * n:(o + d) * n])
                          for i, (o, d) in enumerate(PROJ_FIELDS)], group, device)
    moving.wait()
    summing.wait()
    sh_slice_backward()
    pairs = [(grad_flat[o * n:(o + d) * n], reduced[i]) for i, (o, d) in enumerate(PROJ_FIELDS)]
    pairs.append((grad_flat[11 * n:11 * n + 3 * K * n], coeff_slice.reshape(-1)))
    _coalesced(dist.all_gather_into_tensor, pairs, group, device).wait()


def _all_gather(out, inp, group, async_op=False):
    """all-gather of equal-size contiguous shards into ``out`` (rank-major);
    with ``async_op`` the work handle (wait() before reading ``out``)."""
    if dist.get_backend(group) == "nccl":
        return dist.all_gather_into_tensor(out, inp, group=group, async_op=async_op)
    # gloo has no all_gather_into_tensor
    return dist.all_gather(list(out.chunk(dist.get_world_size(group))), inp, group=group,
                           async_op=async_op)


def exchange_gradients(mode, grad_flat, n, v_colors_local, v_colors_all, sh_backward, group=None,
                       gathering=None):
    """Sum the per-Gaussian gradients of all ranks into ``grad_flat``.

    mode "allreduce": ``grad_flat`` already holds this rank's complete
    gradients; one all-reduce.  mode "gather": ``grad_flat`` holds the
    projection part (v_means without its SH part, v_quats, v_scales,
    v_opacities) and ``v_colors_local`` [C_local, N, 3] the colour
    cotangents.  After the gather, the all-reduce of the projection part
    runs asynchronously while ``sh_backward(v_colors_all)`` writes v_coeffs
    (``grad_flat[11N:]``, outside the reduced range) for all cameras and
    returns the SH part of v_means, which is added once the reduction is
    done.  ``gathering``: the handle of an all-gather of the colour
    cotangents already started (the sharded step starts it before the
    projection backward), waited for instead of gathering here."""
    if mode == "allreduce":
        dist.all_reduce(grad_flat, group=group)
        return
    if mode != "gather":
        raise ValueError(f"unknown exchange {mode!r}")
    if gathering is not None:
        gathering.wait()
    else:
        _all_gather(v_colors_all.view(-1), v_colors_local.reshape(-1), group)
    work = dist.all_reduce(grad_flat[:11 * n], group=group, async_op=True)
    v_means_sh = sh_backward(v_colors_all)
    work.wait()
    grad_flat[:3 * n] += v_means_sh.reshape(-1)


class ShardedTrainingStep:
    """One camera-sharded fwd+bwd step of C_total cameras over the process
    group: this rank renders ``cameras[start:stop]`` and, after the
    exchange, holds the gradient summed over every camera.  All ranks must
    have the same number of cameras (C_total divisible by the world size)."""

    def __init__(self, n, sh_degree, K, cameras_total, width, height, group=None, exchange="auto",
                 heartbeat=None, **step_kw):
        from .pipeline import TrainingStep
        self.group = group
        # liveness.Heartbeat: before a step's first collective every rank
        # must have reached the step (bounded wait, PeerLost otherwise)
        self.heartbeat = heartbeat
        self.steps = 0
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if cameras_total % self.world:
            raise ValueError(f"{cameras_total} cameras do not split evenly over "
                             f"{self.world} ranks")
        self.C_total = int(cameras_total)
        self.start, self.stop = camera_shard(cameras_total, self.world, self.rank)
        self.C = self.stop - self.start
        self.N, self.K, self.deg = int(n), int(K), int(sh_degree)
        self.step = TrainingStep(n, sh_degree, K, self.C, width, height, **step_kw)
        self.exchange = (choose_exchange(self.N, self.K, self.C, self.world)
                         if exchange == "auto" else exchange)
        if self.exchange not in ("allreduce", "gather", "shard"):
            raise ValueError(f"unknown exchange {exchange!r}")
        if self.exchange == "shard" and self.N % self.world:
            raise ValueError(f"the shard exchange needs N ({self.N}) divisible by the "
                             f"{self.world} ranks")
        self.v_colors_all = self.v_means_sh = None
        dev = self.step.dev
        e = lambda *shape: torch.empty(shape, dtype=torch.float32, device=dev)  # noqa: E731
        if self.exchange == "gather" and self.world > 1:
            self.v_colors_all = e(self.C_total, self.N, 3)
            self.v_means_sh = e(self.N, 3)
        if self.exchange == "shard" and self.world > 1:
            ns = self.N // self.world
            self.slice0 = self.rank * ns
            self.recv = e(self.C_total, ns, 3)
            self.reduced = [e(d * ns) for _, d in PROJ_FIELDS]
            self.coeff_slice = e(ns, self.K, 3)


    def local(self, t):
        """This rank's slice of a per-camera tensor [C_total, ...]."""
        return t[self.start:self.stop]

    def run(self, means, quats, scales, opacities, coeffs, viewmats_all, Ks_all,
            v_render_colors, v_render_alphas):
        """``viewmats_all`` / ``Ks_all``: every camera [C_total, 4|3, 4|3];
        ``v_render_*``: this rank's cotangents [C_local, H, W, 3|1].
        Returns (grad_flat summed over all cameras, local intersections)."""
        from .pipeline import sh_colors_backward
        st = self.step
        self.steps += 1
        if self.heartbeat is not None and self.world > 1:
            self.heartbeat.check(self.steps)
        gather = self.exchange == "gather" and self.world > 1
        shard = self.exchange == "shard" and self.world > 1
        gathering = []

        def start_gather():
            # the colour cotangents are final once the rasterizer backward
            # ran: their exchange overlaps the projection backward
            if shard:
                gathering.append(start_shard_all_to_all(self.recv, st.v_colors, self.group))
            else:
                gathering.append(_all_gather(self.v_colors_all.view(-1),
                                             st.v_colors.reshape(-1), self.group, async_op=True))

        flat, m = st.run(means, quats, scales, opacities, coeffs, self.local(viewmats_all),
                         self.local(Ks_all), v_render_colors, v_render_alphas,
                         sh_backward=not (gather or shard),
                         after_raster=start_gather if (gather or shard) else None)
        if self.world == 1:
            return flat, m
        if shard:
            a, b = self.slice0, self.slice0 + self.N // self.world

            def sh_slice():
                sh_colors_backward(self.deg, means[a:b], viewmats_all, coeffs[a:b], None,
                                   self.recv, self.reduced[0].view(-1, 3), radii=None,
                                   v_coeffs=self.coeff_slice, skip_zero_cotangents=True,
                                   camera_groups=self.world)

            shard_exchange(flat, self.N, self.K, self.reduced, self.coeff_slice, sh_slice,
                           gathering[0], self.group, st.dev)
            return flat, m

        def sh_bwd(v_all):
            self.v_means_sh.zero_()
            sh_colors_backward(self.deg, means, viewmats_all, coeffs, None, v_all,
                               self.v_means_sh, radii=None, v_coeffs=st.v_coeffs,
                               skip_zero_cotangents=True)
            return self.v_means_sh

        exchange_gradients("gather" if gather else "allreduce", flat, self.N, st.v_colors,
                           self.v_colors_all, sh_bwd, self.group,
                           gathering=gathering[0] if gathering else None)
        return flat, m

    def gradients(self):
        return self.step.gradients()
