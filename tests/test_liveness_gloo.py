"""Failure detection of the camera-sharded step on CPU ranks (gloo): a rank
that never joins, and a rank that leaves between steps, end the survivors'
waits with an error within a bound instead of a hang.  The failures are made
on the host (a rank that is never started, a rank that exits); no device is
involved."""
from __future__ import annotations

import json
import os
import socket
import time

import pytest
import torch.multiprocessing as mp


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _never_joins(rank, world, port, out):
    import torch.distributed as dist  # noqa: F401
    from gsplat_core.liveness import init_group
    t0 = time.monotonic()
    try:
        init_group("gloo", rank, world, timeout_s=3.0, master_port=port)
        res = {"error": None}
    except Exception as e:  # the missing rank ends the rendezvous
        res = {"error": type(e).__name__}
    res["seconds"] = time.monotonic() - t0
    with open(os.path.join(out, f"nj_{rank}.json"), "w") as f:
        json.dump(res, f)


def _leaves(rank, world, port, out, use_heartbeat):
    import torch
    import torch.distributed as dist
    from gsplat_core.liveness import Heartbeat, PeerLost, abort_group, init_group
    store = init_group("gloo", rank, world, timeout_s=4.0, master_port=port)
    hb = Heartbeat(store, rank, world, deadline_s=1.5)
    x = torch.ones(16)
    # step 1: everybody
    if use_heartbeat:
        hb.check(1)
    dist.all_reduce(x)
    if rank == world - 1:
        os._exit(0)  # leaves between steps, nothing in flight
    t0 = time.monotonic()
    res = {"error": None}
    try:
        if use_heartbeat:
            hb.check(2)
        dist.all_reduce(x)
    except PeerLost as e:
        res = {"error": "PeerLost", "ranks": e.ranks}
    except Exception as e:  # the group's timeout ends the collective
        res = {"error": type(e).__name__}
    res["seconds"] = time.monotonic() - t0
    with open(os.path.join(out, f"lv_{rank}.json"), "w") as f:
        json.dump(res, f)
    if use_heartbeat:
        abort_group()
    os._exit(0)


def _run(target, args_of, ranks, limit):
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=target, args=args_of(r)) for r in ranks]
    t0 = time.monotonic()
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=limit)
        if p.is_alive():
            p.kill()
            pytest.fail("a surviving rank did not return within the limit")
    return time.monotonic() - t0


def test_rank_that_never_joins(tmp_path):
    port = _port()
    # world of three, rank 2 is never started
    _run(_never_joins, lambda r: (r, 3, port, str(tmp_path)), [0, 1], limit=60)
    for r in (0, 1):
        res = json.load(open(tmp_path / f"nj_{r}.json"))
        assert res["error"] is not None, res
        assert res["seconds"] < 30, res


@pytest.mark.parametrize("use_heartbeat", [True, False])
def test_rank_that_leaves_between_steps(tmp_path, use_heartbeat):
    port = _port()
    _run(_leaves, lambda r: (r, 3, port, str(tmp_path), use_heartbeat), [0, 1, 2], limit=60)
    for r in (0, 1):
        res = json.load(open(tmp_path / f"lv_{r}.json"))
        if use_heartbeat:
            # detected on the host before the next collective
            assert res["error"] == "PeerLost" and res["ranks"] == [2], res
            assert res["seconds"] < 5, res
        else:
            # the group's 4 s timeout ends the collective with an error
            assert res["error"] is not None, res
            assert res["seconds"] < 30, res
