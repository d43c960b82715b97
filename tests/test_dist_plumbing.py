"""The N > 1 host plumbing of bench.py on CPU (gloo, world size 2): the
expert-parallel handle exchange returns every rank's bytes in rank order,
and the max / sum reductions used for timing behave as on the GPU box."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank), FC_DIST_BACKEND="gloo")
    sys.path.insert(0, ROOT)
    import bench
    d = bench.Dist()
    handles = d.all_gather_bytes(bytes([rank]) * 64)
    q.put((rank, [h[0] for h in handles], d.max(rank + 1.5), d.sum(rank + 1.0)))
    d.barrier()
    d.close()


def test_gloo_handle_exchange_and_reductions():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 28500 + os.getpid() % 1000
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, firsts, mx, sm in out:
        assert firsts == [0, 1]          # rank order
        assert mx == 2.5 and sm == 3.0


def test_expert_split_matches_single_order():
    """The global slot order is every rank's ascending local slots, rank
    after rank (contiguous expert ranges), so a rank-ordered gather of the
    per-rank outputs is the single-GPU ascending order."""
    import numpy as np
    rng = np.random.default_rng(0)
    E, world = 32, 4
    active = np.sort(rng.choice(E, size=12, replace=False))
    per = E // world
    gathered = []
    for r in range(world):
        gathered += [int(e) for e in active if r * per <= e < (r + 1) * per]
    assert gathered == active.tolist()
