"""Failure detection without any GPU fault: host-side faults between steps
(a rank that stops, a rank that reports an exception, a rank that never
joins) must surface as RankFailure on the surviving rank (gloo, CPU)."""
import os
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from rlx_models_b200.parallel.health import Heartbeat, RankFailure


def _worker(rank, world, port, mode, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
    store = dist.distributed_c10d._get_default_store()
    hb = Heartbeat(store, rank, world, interval=0.1, timeout=1.0)
    t = torch.ones(4)
    dist.all_reduce(t)  # one healthy step
    if rank == 1:
        if mode == "exception":
            hb.report_failure("ValueError in step 2")
        hb.stop()  # mode "exit": the rank stops beating and leaves between steps
        q.put((rank, "left"))
        return
    time.sleep(1.6)
    try:
        hb.check()
        q.put((rank, "no failure detected"))
    except RankFailure as e:
        q.put((rank, f"detected {e.ranks} {e}"))
    hb.stop()


@pytest.mark.parametrize("mode", ["exit", "exception"])
def test_rank_failure_detected(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29950 + (0 if mode == "exit" else 7) + os.getpid() % 20
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=60) for _ in range(2))
    for p in procs:
        p.join(timeout=30)
    assert res[1] == "left"
    assert res[0].startswith("detected [1]"), res[0]
    if mode == "exception":
        assert "ValueError" in res[0]
