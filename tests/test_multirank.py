"""The N > 1 host logic of ``bench.py`` on two CPU ranks (gloo, world size 2).

The path shards by batch row: every rank runs its own batch (same document
layout, so the same work per GPU; its own seeded values) with no data-path
collective (weak scaling); the collectives are the max over ranks of the timed
region and the sum of the ranks' FLOPs, and the job-wide throughput is that sum
over that maximum.  The reference arm prints from rank 0 only.
"""

import io
import os
import socket
import sys
from contextlib import redirect_stdout

import numpy as np
import torch.multiprocessing as mp

from conftest import ROOT


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, out):
    sys.path.insert(0, ROOT)
    import torch.distributed as dist

    import bench

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        t_max = bench.max_over_ranks(1.0 + 0.5 * rank, world, "cpu")
        job = bench.sum_over_ranks(10.0 * (rank + 1), world, "cpu")
        rows, _ = bench.make_rows(seed=0)
        lens = [len(b.query_pos_ids) for b in rows[0]]
        # the reference arm: only rank 0 prints a line
        class A:  # noqa: N801 - argparse stand-in
            steps, warmup = 1, 0
        buf = io.StringIO()
        if rank != 0:
            with redirect_stdout(buf):
                bench.run_reference(A())
        dist.barrier()
        out.put((rank, (t_max, job), lens, buf.getvalue()))
    finally:
        dist.destroy_process_group()


def test_two_ranks_max_timing_and_equal_work():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        rank, t_max, lens, printed = q.get(timeout=120)
        res[rank] = (t_max, lens, printed)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # every rank sees the slowest rank's time and the job's summed FLOPs
    assert res[0][0] == res[1][0] == (1.5, 30.0)
    # the same document layout (so the same work) on every rank
    assert res[0][1] == res[1][1]
    # rank 1 of the reference arm stays silent
    assert res[1][2] == ""


def test_job_tflops_is_weak_scaling():
    sys.path.insert(0, ROOT)
    import bench

    one = bench.job_tflops(1e12, 10, 2.0)
    assert np.isclose(one, 5.0)
    # eight ranks of the same work in the same time: eight times the FLOPs
    assert np.isclose(bench.job_tflops(8 * 1e12, 10, 2.0), 8 * one)
