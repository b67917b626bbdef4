"""Multi-rank host logic on CPU (gloo, world size 2): row sharding with no
data-path collective reproduces the single-process result, and the timing
reduction takes the max over ranks."""
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from kernrt_b200 import workloads as W


def test_shard_rows_partition():
    for total in [0, 1, 7, 65536, 65537]:
        for world in [1, 2, 3, 4, 8]:
            spans = [W.shard_rows(total, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [hi - lo for lo, hi in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        W.shard_rows(10, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _inputs(rows, wl):
    rng = np.random.default_rng(3)
    from oracle import oracle

    table = oracle.f32_to_bf16_bits(rng.standard_normal((64, wl.dim), dtype=np.float32) * 0.02)
    return dict(table=table, tokens=rng.integers(0, 64, rows).astype(np.int32),
                w=(1 + 0.1 * rng.standard_normal(wl.dim)).astype(np.float32),
                q=rng.standard_normal((rows, wl.q_dim), dtype=np.float32),
                k=rng.standard_normal((rows, wl.kv_dim), dtype=np.float32),
                gate=rng.standard_normal((rows, wl.hidden), dtype=np.float32),
                up=rng.standard_normal((rows, wl.hidden), dtype=np.float32),
                resid=rng.standard_normal((rows, wl.dim), dtype=np.float32))


def _run_rows(d, lo, hi, wl):
    from oracle import oracle

    return oracle.chain(dim=wl.dim, q_dim=wl.q_dim, kv_dim=wl.kv_dim, hidden=wl.hidden, head=wl.head,
                        eps=wl.eps, theta=wl.theta, positions=wl.positions(lo, hi).astype(np.uint64),
                        w_att=d["w"], q=d["q"][lo:hi], k=d["k"][lo:hi], gate=d["gate"][lo:hi],
                        up=d["up"][lo:hi], resid=d["resid"][lo:hi], tokens=d["tokens"][lo:hi],
                        table=(oracle.BF16, d["table"], None, 64))


def _worker(rank, world, port, rows, q):
    import torch

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        wl = W.Workload("shard", 64, 64, 4, 2, 16, 96, 1e4, 1e-5, "bf16", rows=rows, seq_len=13)
        d = _inputs(rows, wl)
        lo, hi = W.shard_rows(rows, world, rank)
        out = _run_rows(d, lo, hi, wl)
        mine = np.concatenate([out[n].ravel() for n in ["x", "xb", "q", "k", "gate"]])
        gathered = [None] * world
        dist.all_gather_object(gathered, (lo, hi, mine))
        t = torch.tensor([float(rank + 1)], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        if rank == 0:
            q.put((gathered, float(t.item())))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(120)
def test_two_rank_row_shards_reassemble_the_whole_batch():
    rows, world = 37, 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, rows, q)) for r in range(world)]
    for p in procs:
        p.start()
    gathered, tmax = q.get(timeout=100)
    for p in procs:
        p.join(timeout=30)
        assert p.exitcode == 0
    assert tmax == float(world)
    wl = W.Workload("shard", 64, 64, 4, 2, 16, 96, 1e4, 1e-5, "bf16", rows=rows, seq_len=13)
    d = _inputs(rows, wl)
    full = _run_rows(d, 0, rows, wl)
    for lo, hi, flat in gathered:
        part = _run_rows(d, lo, hi, wl)
        want = np.concatenate([part[n].ravel() for n in ["x", "xb", "q", "k", "gate"]])
        assert np.array_equal(flat.view(np.uint32), want.view(np.uint32))
        for n in ["x", "xb", "q", "k", "gate"]:
            assert np.array_equal(part[n].view(np.uint32), full[n][lo:hi].view(np.uint32))
