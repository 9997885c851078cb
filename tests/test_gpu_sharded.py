"""Camera-sharded step on two GPUs (NCCL): every gradient exchange gives the
gradients of one single-GPU TrainingStep over all cameras.  Skipped where
fewer than two GPUs are visible."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _scene():
    from gsplat_core import synthetic as S
    sc = S.config3(seed=4, n=200_000)
    C = 4
    sc.viewmats = S.orbit(C, 4.0)
    sc.Ks = np.repeat(sc.Ks[:1], C, 0).copy()
    sc.Ks[:, :2, :] /= 2
    sc.width, sc.height = sc.width // 2, sc.height // 2
    vrc, vra = S.cotangents(6, C, sc.height, sc.width)
    return sc, vrc, vra


def _args(sc, dev, torch):
    T = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(dev)  # noqa: E731
    return [T(sc.means), T(sc.quats), T(sc.scales), T(sc.opacities), T(sc.coeffs),
            T(sc.viewmats), T(sc.Ks)]


def _worker(rank, world, port, mode, out_dir):
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=dev)
    try:
        from gsplat_core.sharded import ShardedTrainingStep
        sc, vrc, vra = _scene()
        st = ShardedTrainingStep(sc.n, 3, 16, sc.cameras, sc.width, sc.height, exchange=mode,
                                 device=dev)
        args = _args(sc, dev, torch)
        T = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(dev)  # noqa: E731
        flat, _ = st.run(*args, T(st.local(vrc)), T(st.local(vra)))
        torch.cuda.synchronize()
        np.save(os.path.join(out_dir, f"{mode}_{rank}.npy"), flat.cpu().numpy())
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["allreduce", "gather", "shard"])
def test_two_gpu_exchange_matches_single_gpu(gs, cuda, tmp_path, mode):
    import torch
    import torch.multiprocessing as mp
    from _util import assert_grad_close
    from gsplat_core import pipeline
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from test_gpu_chain import oracle_step
    sc, vrc, vra = _scene()
    step = pipeline.TrainingStep(sc.n, 3, 16, sc.cameras, sc.width, sc.height)
    T = lambda x: torch.from_numpy(np.ascontiguousarray(x)).cuda()  # noqa: E731
    flat, _ = step.run(*_args(sc, torch.device("cuda", 0), torch), T(vrc), T(vra))
    single = flat.cpu().numpy()
    # the oracle's gradients, with the spread another summation order gives
    # them (sums over 4 cameras with heavy cancellation on some entries)
    from oracle.oracle import Oracle
    e = oracle_step(Oracle(), sc, np.arange(sc.n), vrc, vra, noise=True)
    keys = ("v_means", "v_quats", "v_scales", "v_opacities", "v_coeffs")
    expect = np.concatenate([e["grads"][k].ravel() for k in keys])
    noise = np.concatenate([e["noise"][k].ravel() for k in keys])
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        if p.is_alive():
            p.kill()
            pytest.fail("a rank did not finish")
        assert p.exitcode == 0
    outs = [np.load(tmp_path / f"{mode}_{r}.npy") for r in range(2)]
    np.testing.assert_array_equal(outs[0], outs[1])
    n = sc.n
    for name, a, b in (("v_means", 0, 3 * n), ("v_quats", 3 * n, 7 * n),
                       ("v_scales", 7 * n, 10 * n), ("v_opacities", 10 * n, 11 * n),
                       ("v_coeffs", 11 * n, expect.size)):
        for what, got in ((f"{mode} {name}", outs[0]), (f"one GPU {name}", single)):
            assert_grad_close(got[a:b], expect[a:b], what, atol_frac=1e-4, noise=noise[a:b])


def _leaver(rank, world, port, out_dir):
    """NCCL ranks on their own GPUs; the last rank leaves after step 1 with
    nothing in flight; the others must learn it on the host (heartbeat)
    before step 2's collective and abort their communicators."""
    import json
    import time
    import torch
    import torch.distributed as dist
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    from gsplat_core.liveness import Heartbeat, PeerLost, abort_group, init_group
    store = init_group("nccl", rank, world, timeout_s=20.0, device=dev, master_port=port)
    hb = Heartbeat(store, rank, world, deadline_s=2.0)
    x = torch.ones(1 << 16, device=dev)
    hb.check(1)
    dist.all_reduce(x)
    torch.cuda.synchronize()
    if rank == world - 1:
        os._exit(0)
    t0 = time.monotonic()
    res = {"error": None}
    try:
        hb.check(2)
        dist.all_reduce(x)
        torch.cuda.synchronize()
    except PeerLost as e:
        res = {"error": "PeerLost", "ranks": e.ranks}
    res["seconds"] = time.monotonic() - t0
    abort_group()
    with open(os.path.join(out_dir, f"leave_{rank}.json"), "w") as f:
        json.dump(res, f)
    os._exit(0)


def test_two_gpu_rank_leaving_is_detected(gs, cuda, tmp_path):
    import json
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_leaver, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
            pytest.fail("the surviving rank did not return")
    res = json.load(open(tmp_path / "leave_0.json"))
    assert res["error"] == "PeerLost" and res["ranks"] == [1], res
    assert res["seconds"] < 10, res
