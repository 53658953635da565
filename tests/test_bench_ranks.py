"""CPU: the benchmark's multi-rank host logic on world-size-2 gloo ranks --
stream sharding (independent streams, no data-path collective), the start
barrier and the max / sum reductions of the per-rank timings."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench():
    if ROOT not in sys.path:
        sys.path.insert(0, ROOT)
    import bench
    return bench


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_shard_partitions_streams(world):
    bench = _bench()
    parts = [bench.shard(r, world, 64) for r in range(world)]
    assert all(len(p) == 64 // world for p in parts)
    assert sorted(s for p in parts for s in p) == list(range(64))


def _rank(rank, world, port, out):
    import torch
    import torch.distributed as dist
    bench = _bench()
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        assert bench.dist_env() == (rank, world, rank)
        bench.barrier(world)
        dev = torch.device("cpu")
        out.put((rank, bench.reduce_over_ranks(1.5 + rank, world, dev, "max"),
                 bench.reduce_over_ranks(1.5 + rank, world, dev, "sum"), bench.shard(rank, world, 64)))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks():
    import socket
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    got = sorted(q.get(timeout=5) for _ in range(2))
    assert [g[1] for g in got] == [2.5, 2.5]   # max over ranks
    assert [g[2] for g in got] == [4.0, 4.0]   # sum over ranks
    assert got[0][3] == list(range(32)) and got[1][3] == list(range(32, 64))
