"""Failure detection on host ranks (gloo, CPU): a rank that dies or leaves between updates is
detected by the others within a bounded time, by the heartbeat before their next launch and by
the process group's collective timeout.  No GPU is involved."""
import os
import time

import torch
import torch.multiprocessing as mp

from tests.conftest import free_port


def _worker(rank, port, mode, results):
    from datetime import timedelta
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), CUDA_VISIBLE_DEVICES="")
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=timedelta(seconds=10))
    from nexttransformer_b200.runtime.liveness import Heartbeat, RankFailure
    hb = Heartbeat()
    t = torch.ones(4)
    for step in range(3):
        if rank == 1 and step == 2:
            if mode == "leave":
                hb.leave()
            os._exit(0)      # between updates: no kernel or collective of this rank is in flight
        hb.beat(step)
        t0 = time.monotonic()
        try:
            hb.wait_peers(step, timeout_s=3.0)
        except RankFailure as exc:
            results["detected"] = (step, exc.ranks, time.monotonic() - t0)
            break
        dist.all_reduce(t)
    if rank == 0:
        # the collective with the missing rank also ends with an error, within the group timeout
        t0 = time.monotonic()
        try:
            dist.all_reduce(t)
            results["collective"] = ("completed", time.monotonic() - t0)
        except Exception as exc:  # noqa: BLE001 - gloo raises RuntimeError or DistBackendError
            results["collective"] = (type(exc).__name__, time.monotonic() - t0)
    os._exit(0)


def _run(mode):
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        results = m.dict()
        port = free_port()
        procs = [ctx.Process(target=_worker, args=(r, port, mode, results)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=120)
            assert p.exitcode is not None, "a rank did not finish"
        return dict(results)


def test_dead_rank_is_detected_by_heartbeat_and_collective_timeout():
    res = _run("die")
    step, ranks, waited = res["detected"]
    assert step == 2 and ranks == [1] and waited < 10
    kind, waited = res["collective"]
    assert kind != "completed" and waited < 60


def test_leaving_rank_is_detected_at_once():
    res = _run("leave")
    step, ranks, waited = res["detected"]
    assert step == 2 and ranks == [1] and waited < 1.5
