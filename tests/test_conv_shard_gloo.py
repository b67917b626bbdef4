"""The LFM2 short-conv block split across ranks on sequence rows (CPU, gloo).

A rank's contiguous rows may start inside a sequence; the causal conv then
needs the k - 1 rows of that sequence before them.  Each rank stages those
halo rows with its own (a local copy taken before the run: no remote reads on
the data path), computes its segments with the oracle, and the gathered
results must equal the unsharded block bit for bit, the decode ring too
(lfm2.rs:584-624, ring seeding :601-610).  The device form of the halo is
checked against the same oracle by tests/test_gpu_rowops.py.
"""
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from kernrt_b200 import workloads as W

DIM, K = 48, 3


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _sequences(seq_lens, seed=21):
    rng = np.random.default_rng(seed)
    bcx = [rng.standard_normal((n, 3 * DIM), dtype=np.float32) for n in seq_lens]
    kernel = (0.3 * rng.standard_normal((DIM, K))).astype(np.float32)
    return bcx, kernel


def _rank_segments(seq_lens, world, rank):
    """This rank's (sequence, lo, hi, cy, ring or None), from its own rows and
    their staged halo only."""
    from oracle import oracle

    bcx, kernel = _sequences(seq_lens)
    out = []
    for seq, lo, hi, halo, ends in W.conv_shards(seq_lens, world, rank, K):
        staged = bcx[seq][lo - halo:hi].copy()  # the rank's rows and its halo, local before the run
        cy, ring = oracle.lfm2_conv_block_shard(staged, kernel, K, halo, halo + (hi - lo), halo)
        out.append((seq, lo, hi, cy, ring if ends else None))
    return out


def _worker(rank, world, port, seq_lens, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mine = _rank_segments(seq_lens, world, rank)
        gathered = [None] * world
        dist.all_gather_object(gathered, mine)
        if rank == 0:
            q.put(gathered)
    finally:
        dist.destroy_process_group()


def _check(seq_lens, gathered):
    from oracle import oracle

    bcx, kernel = _sequences(seq_lens)
    full = [oracle.lfm2_conv_block(b, kernel, np.zeros((K - 1, DIM), np.float32), K) for b in bcx]
    covered = [np.zeros(n, bool) for n in seq_lens]
    rings = {}
    for segs in gathered:
        for seq, lo, hi, cy, ring in segs:
            want = full[seq][0][lo:hi]
            assert np.array_equal(cy.view(np.uint32), want.view(np.uint32)), f"sequence {seq} rows {lo}:{hi}"
            covered[seq][lo:hi] = True
            if ring is not None:
                rings[seq] = ring
    assert all(c.all() for c in covered)
    for seq in range(len(seq_lens)):
        assert np.array_equal(rings[seq].view(np.uint32), full[seq][1].view(np.uint32)), f"ring of {seq}"


def test_conv_shard_plan_covers_every_row_once():
    for seq_lens in ([1024], [100, 50, 200], [1, 2, 3], [7]):
        for world in (1, 2, 3, 4, 8):
            seen = [np.zeros(n, int) for n in seq_lens]
            for r in range(world):
                for seq, lo, hi, halo, ends in W.conv_shards(seq_lens, world, r, K):
                    seen[seq][lo:hi] += 1
                    assert halo == min(K - 1, lo) and ends == (hi == seq_lens[seq])
            assert all((s == 1).all() for s in seen)


@pytest.mark.parametrize("world", [2, 3, 4])
def test_sharded_conv_block_in_process(world):
    seq_lens = [100, 50, 200]
    _check(seq_lens, [_rank_segments(seq_lens, world, r) for r in range(world)])


@pytest.mark.timeout(120)
def test_two_rank_conv_shards_reassemble_the_sequence():
    seq_lens, world = [1024], 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, seq_lens, q)) for r in range(world)]
    for p in procs:
        p.start()
    gathered = q.get(timeout=100)
    for p in procs:
        p.join(timeout=30)
        assert p.exitcode == 0
    _check(seq_lens, gathered)
