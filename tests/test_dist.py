"""Multi-rank host logic of bench.py on CPU (gloo, world size 2): the max-over-
ranks timing reduction and the whole-job throughput.  The path shards by
(batch, head) with no data-path collective, so this is the only cross-rank logic."""
import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import bench
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        t = bench.max_over_ranks(10.0 + 5.0 * rank)
        v = bench.aggregate_tflops(68.75e9, world, t / 100)
        q.put((rank, t, v))
    finally:
        dist.destroy_process_group()


def test_max_over_ranks_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert [r[1] for r in res] == [15.0, 15.0]
    assert res[0][2] == pytest.approx(68.75e9 * 2 / (0.15e-3) / 1e12)


def test_single_process_identity():
    import bench
    assert bench.max_over_ranks(3.5) == 3.5
    assert bench.aggregate_tflops(1e12, 1, 1000.0) == pytest.approx(1.0)
