"""bench.py's multi-replica aggregation on two gloo ranks (CPU, no GPU): every rank learns the slowest rank's time
and the whole-job rate counts all ranks' units over that time."""
import os
import socket
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, ws, port, out):
    import datetime

    import torch.distributed as dist

    sys.path.insert(0, ROOT)
    import bench

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=ws, timeout=datetime.timedelta(seconds=60))
    try:
        ms = bench.max_over_ranks(10.0 + 5.0 * rank, dist, "cpu")
        rate = bench.whole_job_rate(ws, 306 * 4, ms / 1000)
        out.put((rank, ms, rate))
    finally:
        dist.destroy_process_group()


def test_two_rank_max_and_rate():
    torch = pytest.importorskip("torch")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert [r[1] for r in res] == [15.0, 15.0]
    assert all(abs(r[2] - 2 * 306 * 4 / 0.015) < 1e-6 for r in res)


def test_single_rank_is_identity():
    sys.path.insert(0, ROOT)
    import bench

    assert bench.max_over_ranks(3.5, None, "cpu") == 3.5
    assert bench.whole_job_rate(1, 100, 0.5) == 200.0
