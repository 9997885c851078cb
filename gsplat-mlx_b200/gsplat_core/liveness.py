"""Failure detection for the camera-sharded step: bounded waits on the host.

A rank that never joins, or that leaves between steps, must not leave the
others waiting in a collective for ever.  Three bounds:

* ``init_group`` creates the process group with a short timeout: the
  rendezvous gives up when a rank never joins, and every collective fails
  (instead of hanging) once it waits longer than the timeout.  With NCCL the
  communicator is created in nonblocking mode (``ncclCommInitRankConfig``
  with ``blocking = 0``), so that its initialisation is bounded by the same
  host-side deadline, and a failed group is aborted (``ncclCommAbort``
  through the process group's abort) rather than destroyed with work in
  flight.
* ``Heartbeat`` publishes each rank's step count in the rendezvous store;
  ``Heartbeat.check(step)`` is called before a step's first collective and
  raises ``PeerLost`` (naming the silent ranks) when a peer has not reached
  the step within ``deadline_s``.  A rank leaves only between steps, with
  none of its kernels or collectives in flight, so the survivors learn of it
  on the host before they launch anything that would wait for it.
* ``abort_group`` tears the group down after ``PeerLost`` or a collective
  timeout.

The reference has no distributed path (its validation is ``throw
std::runtime_error`` in the operator front-ends); this is the
bounded-wait part of the multi-GPU path built here.
"""
from __future__ import annotations

import time
from datetime import timedelta

import torch.distributed as dist


class PeerLost(RuntimeError):
    """Peers that did not reach a step within the deadline."""

    def __init__(self, step, ranks):
        super().__init__(f"ranks {sorted(ranks)} did not reach step {step} in time")
        self.step = step
        self.ranks = sorted(ranks)


def init_group(backend, rank, world, timeout_s=30.0, device=None, master_addr="127.0.0.1",
               master_port=None):
    """Process group with a ``timeout_s`` bound on the rendezvous and on
    every collective; NCCL communicators are created nonblocking.  Raises
    (instead of hanging) when a rank does not join in time.  Returns the
    store (for ``Heartbeat``)."""
    import os
    if master_port is not None:
        os.environ["MASTER_ADDR"] = master_addr
        os.environ["MASTER_PORT"] = str(master_port)
    timeout = timedelta(seconds=float(timeout_s))
    store = dist.TCPStore(os.environ.get("MASTER_ADDR", master_addr),
                          int(os.environ["MASTER_PORT"]), world, rank == 0, timeout=timeout,
                          wait_for_workers=False)
    kw = dict(backend=backend, store=store, rank=rank, world_size=world, timeout=timeout)
    if backend == "nccl":
        from torch.distributed import ProcessGroupNCCL
        opts = ProcessGroupNCCL.Options()
        opts.config.blocking = 0  # nonblocking communicator creation
        kw["pg_options"] = opts
        if device is not None:
            kw["device_id"] = device
    dist.init_process_group(**kw)
    # the rendezvous above returns before every rank is in: a barrier with
    # the group's timeout proves they all are
    dist.barrier()
    return store


class Heartbeat:
    """Step counts of all ranks in the store.  ``beat(step)`` marks this
    rank as having reached ``step``; ``check(step)`` waits at most
    ``deadline_s`` for every rank to mark it and raises PeerLost otherwise."""

    def __init__(self, store, rank, world, deadline_s=5.0, poll_s=0.005, prefix="gsplat_hb"):
        self.store, self.rank, self.world = store, int(rank), int(world)
        self.deadline_s, self.poll_s, self.prefix = float(deadline_s), float(poll_s), prefix

    def _key(self, r):
        return f"{self.prefix}/{r}"

    def beat(self, step):
        self.store.set(self._key(self.rank), str(int(step)))

    def reached(self, r):
        try:
            return int(self.store.get(self._key(r)).decode())
        except Exception:  # key absent: the rank never beat
            return -1

    def check(self, step):
        """Marks ``step`` and waits (bounded) until every rank marked it."""
        self.beat(step)
        end = time.monotonic() + self.deadline_s
        missing = set(range(self.world)) - {self.rank}
        while True:
            missing = {r for r in missing if not self.store.check([self._key(r)])
                       or self.reached(r) < step}
            if not missing:
                return
            if time.monotonic() >= end:
                raise PeerLost(step, missing)
            time.sleep(self.poll_s)


def abort_group(group=None):
    """Tears the process group down after a lost peer or a timed-out
    collective: NCCL communicators are aborted (no waiting on work that
    can no longer finish), other backends destroyed."""
    if not dist.is_initialized():
        return
    try:
        pg = group or dist.group.WORLD
        if dist.get_backend(pg) == "nccl" and hasattr(pg, "abort"):
            pg.abort()
    finally:
        try:
            dist.destroy_process_group(group)
        except Exception:
            pass
