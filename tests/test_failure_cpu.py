"""CPU: a rank that leaves a multi-GPU job between steps is detected on the
host, before the next step launches anything.

Two gloo ranks (world_size 2, 127.0.0.1) run steps; each step begins with
partition.Heartbeat.beat(step) and then an all-reduce standing in for the
step's collective.  Rank 1 runs step 0 and exits.  Rank 0 must see PeerLost
at step 1 within the heartbeat timeout, without entering the collective
(which would otherwise wait for the missing rank).  The reference has no
multi-rank path; its failure handling is decline-then-fallback
(zblas/zblas_gpu.cpp:184-201).
"""
import os
import socket
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out):
    import sys
    sys.path.insert(0, ROOT)
    from datetime import timedelta
    import torch
    import torch.distributed as dist
    from zlift_b200.partition import Heartbeat, PeerLost
    store = dist.TCPStore("127.0.0.1", port, world, rank == 0, timedelta(seconds=30))
    dist.init_process_group("gloo", store=store, rank=rank, world_size=world,
                            timeout=timedelta(seconds=30))
    hb = Heartbeat(store, world, rank, timeout_s=1.0)
    log = []
    try:
        for step in range(3):
            if rank == 1 and step == 1:
                log.append("left")
                break                      # leaves between steps, nothing in flight
            t0 = time.perf_counter()
            try:
                hb.beat(step)
            except PeerLost as e:
                log.append(("lost", step, round(time.perf_counter() - t0, 2), str(e)))
                break
            x = torch.ones(4)
            dist.all_reduce(x)             # the step's collective
            log.append(("step", step, float(x[0])))
    finally:
        out[rank] = log
        if rank == 0:
            # keep the store up until the other rank is gone for sure
            time.sleep(0.2)
        os._exit(0)                        # no group teardown with a lost peer


def test_rank_leaving_between_steps_is_seen_before_next_launch():
    import torch.multiprocessing as mp
    world = 2
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    out = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    log0, log1 = out[0], out[1]
    assert log1 == [("step", 0, 2.0), "left"]
    assert log0[0] == ("step", 0, 2.0)
    kind, step, waited, msg = log0[1]
    assert kind == "lost" and step == 1
    assert waited < 10.0
    assert "1" in msg
    assert len(log0) == 2                  # no collective of step 1 was entered


def test_heartbeat_single_rank_never_waits():
    from datetime import timedelta
    import torch.distributed as dist
    from zlift_b200.partition import Heartbeat
    store = dist.HashStore()
    hb = Heartbeat(store, 1, 0, timeout_s=0.1)
    for step in range(3):
        hb.beat(step)
    assert store.check(["hb/2/0"])
    _ = timedelta
