"""The multi-GPU path's host logic on two CPU ranks (gloo): each rank takes
its own pages (weak scaling, no data-path collective), and the bench's
whole-job number is every rank's pages over the slowest rank's time. The
ranks rendezvous on 127.0.0.1."""

from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import numpy as np
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def rank_main(rank: int, world: int, port: int, out):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    sys.path.insert(0, str(ROOT))
    import bench

    d = bench.Dist()
    d.init("gloo")
    try:
        workload = bench.package().workload
        page = workload.Page(seed=1000 + d.rank, det_size=(64, 48), lines=3)  # the bench's per-rank pages
        d.barrier()
        # rank r "took" (r + 1) seconds for its 4 pages
        value, slowest = d.whole_job(4, float(rank + 1))
        out.put((rank, float(page.det.sum()), value, slowest, d.max(float(10 * rank))))
    finally:
        d.close()


def test_two_ranks_shard_pages_and_take_the_slowest_time():
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=rank_main, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    results = sorted(out.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    (r0, sum0, v0, t0, m0), (r1, sum1, v1, t1, m1) = results
    assert (r0, r1) == (0, 1)
    assert not np.isclose(sum0, sum1)  # each rank its own page
    assert t0 == t1 == 2.0             # the slowest rank's time on both
    assert v0 == v1 == 2 * 4 / 2.0     # all ranks' pages over it
    assert m0 == m1 == 10.0
