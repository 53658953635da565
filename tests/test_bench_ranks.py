"""CPU: the benchmark's multi-rank host logic on world-size-2 gloo ranks --
stream sharding (independent streams, no data-path collective), the start
barrier and the max / sum reductions of the per-rank timings -- and its
per-launch roofline arithmetic."""
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


def test_launch_rooflines_take_each_launchs_slower_bound():
    """The per-launch roofline: every convolution launch is bounded by the
    slower of its int8 MMA time at the peak and its DRAM bytes at the copy
    bandwidth; depthwise launches are reported against the copy bandwidth."""
    bench = _bench()
    peak_tops, hbm_gbs = 4000.0, 5000.0
    table = {
        # 1e12 int16 MACs: 8e12 int8 ops -> 2 ms at 4000 TOPS; 1 GB -> 0.2 ms: tensor-bound
        "conv 512>512 1x1 +res @ 100": [10, 1e12, 4.0, 1e9],
        # 1e10 MACs -> 0.02 ms; 10 GB -> 2 ms: DRAM-bound
        "conv 256>256 1x1 +lut @ 100": [10, 1e10, 4.0, 1e10],
        "depthwise 256 3x3 @ 100": [5, 1e9, 2.0, 5e9],
    }
    conv, depth = bench.launch_rooflines(table, peak_tops, hbm_gbs, step_ms=20.0)
    assert conv["floor_ms"] == pytest.approx(4.0)
    assert conv["measured_ms"] == pytest.approx(8.0)
    assert conv["frac"] == pytest.approx(0.5)
    assert conv["hbm_bound_time_share"] == pytest.approx(0.5)
    assert depth["launches"] == 5
    assert depth["share_of_serial_step"] == pytest.approx(0.1)
    assert depth["achieved_gbs"] == pytest.approx(2500.0)
    assert depth["frac"] == pytest.approx(0.5)
    conv, depth = bench.launch_rooflines({k: v for k, v in table.items() if k.startswith("conv")},
                                         peak_tops, hbm_gbs, step_ms=20.0)
    assert depth is None
