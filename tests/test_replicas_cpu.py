"""The N > 1 path of bench.py on CPU: two gloo ranks, each timing its own replica, agree on the
whole-job duration (max over ranks) and the aggregate throughput; replicas exchange nothing else."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank(rank, ws, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=ws, timeout=datetime.timedelta(seconds=60))
    import bench
    local_ms = [120.0, 95.0, 130.0, 101.0][rank]
    total = bench.max_over_ranks(local_ms, ws)
    value = bench.job_throughput(ws, 10, total)
    dist.barrier()
    dist.destroy_process_group()
    q.put((rank, total, value))


@pytest.mark.parametrize("ws", [2, 4])
def test_max_over_ranks_and_job_throughput(ws):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, ws, port, q)) for r in range(ws)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(ws)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    expect = max([120.0, 95.0, 130.0, 101.0][:ws])
    for _, total, value in res:
        assert total == expect
        assert value == pytest.approx(ws * 10 / (expect / 1000.0))


def test_single_rank_needs_no_process_group():
    import bench
    assert bench.max_over_ranks(12.5, 1) == 12.5
    assert bench.job_throughput(1, 20, 500.0) == pytest.approx(40.0)
