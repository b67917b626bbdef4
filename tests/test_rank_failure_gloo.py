"""A rank that leaves between steps is reported by the survivors on the host,
within a bounded time, before they launch the next step (CPU, gloo, world
size 2; no GPU is involved, so no device is left waiting on the dead rank)."""
import datetime
import os
import socket
import time

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from kernrt_b200.ranks import RankFailure, StepWatch


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q, leave_after):
    import torch

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    watch = StepWatch(dist.distributed_c10d._get_default_store(), rank, world, timeout_s=3.0)
    done = []
    try:
        for step in range(3):
            if rank == 1 and step == leave_after:
                os._exit(0)  # leaves between steps: no collective of this step was entered
            watch.enter(f"step{step}")
            t = torch.tensor([float(rank + 1)])
            dist.all_reduce(t)  # the step's own collective (the timing max in bench.py)
            done.append(step)
        q.put((rank, "finished", done))
    except RankFailure as e:
        q.put((rank, "failure", (e.step, e.missing, done)))
    q.close()
    q.join_thread()  # the report is on its way before the process ends
    os._exit(0)  # a peer may be gone: skip the process group's shutdown handshake


@pytest.mark.timeout(120)
def test_survivor_reports_a_rank_that_left_between_steps():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    t0 = time.time()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, 1)) for r in range(world)]
    for p in procs:
        p.start()
    rank, kind, detail = q.get(timeout=90)
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert (rank, kind) == (0, "failure"), (rank, kind, detail)
    step, missing, done = detail
    assert step == "step1" and missing == [1] and done == [0]
    assert time.time() - t0 < 90


@pytest.mark.timeout(120)
def test_step_watch_passes_when_every_rank_arrives():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, 99)) for r in range(world)]
    for p in procs:
        p.start()
    got = sorted(q.get(timeout=90) for _ in range(world))
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert got == [(0, "finished", [0, 1, 2]), (1, "finished", [0, 1, 2])]
