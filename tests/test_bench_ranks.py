"""The multi-process host logic of bench.py on CPU: two gloo ranks, as torchrun starts
them on a GPU box (one process per GPU).  Every rank runs its own batch (no data-path
collective); the step time that counts is the slowest rank's, and the whole-job rate
is world_size x batch x steps over that time."""
import os
import socket
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, ws, port, out):
    import datetime

    import torch.distributed as dist
    sys.path.insert(0, ROOT)
    import bench
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=ws,
                            timeout=datetime.timedelta(seconds=60))
    try:
        local_ms = 10.0 + 5.0 * rank   # rank 1 is the slower one
        ms = bench.max_over_ranks(local_ms, ws, "cpu")
        out.put((rank, ms, bench.job_rate(ws, 256, 50, ms * 1e-3)))
    finally:
        dist.destroy_process_group()


def test_max_over_ranks_and_job_rate_gloo():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    got = sorted(q.get(timeout=10) for _ in range(2))
    for rank, ms, rate in got:
        assert ms == 15.0                       # the slowest rank's time, on both ranks
        assert rate == pytest.approx(2 * 256 * 50 / 0.015)


def test_single_rank_needs_no_process_group():
    sys.path.insert(0, ROOT)
    import bench
    assert bench.max_over_ranks(3.5, 1, "cpu") == 3.5
    assert bench.job_rate(1, 256, 10, 2.0) == 1280.0
