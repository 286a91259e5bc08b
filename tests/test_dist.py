"""Multi-rank host logic on CPU (gloo): the (batch, head) partition of one forward
across ranks, the optional all-gather that reassembles O / LSE, bench.py's
max-over-ranks timing reduction and its whole-job throughput."""
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


def _stand_in_forward(q, k, v, out=None, lse_out=None):
    """Per-head arithmetic standing in for the attention forward on CPU: any function
    that treats each (b, h) independently checks the partition and the reassembly."""
    o = q * 2.0 + k - v
    lse = q.sum(-1) - v.amax(-1)
    if out is not None:
        out.copy_(o)
        lse_out.copy_(lse)
        return out, lse_out
    return o, lse


def _worker(rank, world, port, BH, q_out):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import bench
    from polyhedral_b200 import shard
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # the same seeded full-size inputs on every rank; each runs only its heads
        g = torch.Generator().manual_seed(7)
        q, k, v = (torch.randn(BH, 16, 8, generator=g) for _ in range(3))
        sh = shard.shard_bh(BH, rank, world)
        o_loc, l_loc = sh.run(_stand_in_forward, q, k, v)
        assert o_loc.shape[0] == sh.size
        o, lse = shard.gather(o_loc, l_loc, sh)
        o_ref, l_ref = _stand_in_forward(q, k, v)
        same = bool(torch.equal(o, o_ref) and torch.equal(lse, l_ref))
        # the forward written into full-size outputs touches only this rank's rows
        out = torch.full((BH, 16, 8), float("nan"))
        lout = torch.full((BH, 16), float("nan"))
        sh.run(_stand_in_forward, q, k, v, out=out, lse_out=lout)
        rows = (~torch.isnan(out[:, 0, 0])).nonzero().flatten().tolist()
        t = bench.max_over_ranks(10.0 + 5.0 * rank)
        q_out.put((rank, sh.start, sh.stop, same, rows, t))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,BH", [(2, 128), (2, 5), (3, 16)])
def test_head_shards_gloo(world, BH):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, BH, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=180) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # contiguous ranges covering [0, BH) exactly once, in rank order
    covered = []
    for rank, start, stop, same, rows, t in res:
        covered.extend(range(start, stop))
        assert same, f"rank {rank}: gathered result differs from the unsharded one"
        assert rows == list(range(start, stop))
        assert t == 10.0 + 5.0 * (world - 1)
    assert covered == list(range(BH))


def test_shard_bh_partition():
    from polyhedral_b200 import shard
    for BH in (1, 7, 128):
        for world in (1, 2, 3, 8):
            if world > BH:
                continue
            parts = [shard.shard_bh(BH, r, world) for r in range(world)]
            assert parts[0].start == 0 and parts[-1].stop == BH
            assert all(a.stop == b.start for a, b in zip(parts, parts[1:]))
            sizes = [p.size for p in parts]
            assert max(sizes) - min(sizes) <= 1
    assert shard.shard_bh(128, 7, 8).start == 112 and shard.shard_bh(128, 7, 8).size == 16
    with pytest.raises(ValueError):
        shard.shard_bh(16, 2, 2)


def test_single_process_identity():
    import bench
    assert bench.max_over_ranks(3.5) == 3.5
    assert bench.job_tflops(1e12, 1000.0) == pytest.approx(1.0)


def test_bench_config_same_for_both_arms():
    """Both arms print one config object for a workload: the one config_of returns."""
    import bench
    for wl in bench.WORKLOADS:
        for world in (1, 8):
            c = bench.config_of(wl, world)
            B, H, N, D = bench.WORKLOADS[wl][:4]
            assert c["global_batch"] == B * H and c["seq_len"] == N and c["head_dim"] == D
            assert "parallelism" in c and "l2" in c
    assert bench.DEFAULT_WORKLOAD == "c5"
