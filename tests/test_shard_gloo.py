"""Multi-process host logic of the sharded benchmark on CPU (gloo, world_size 2): shard seeds partition one big
run exactly, and the timing reduction takes the max over ranks."""
import os
import socket

import pytest
import torch.multiprocessing as mp
from conftest import fme  # noqa: F401  (registers the package)

from fast_mario_env_b200 import shard


def test_shards_partition_the_single_run_streams():
    n, world, seed = 5, 3, 7
    merged = sum((shard.shard_seeds(seed, r, n) for r in range(world)), [])
    assert merged == [seed * 1000 + i for i in range(n * world)]
    assert shard.env_offset(2, 4096) == 8192
    assert shard.job_throughput(8, 1000, 10, 500.0) == 8 * 1000 * 10 / 0.5


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        ms = 100.0 + 50.0 * rank
        got = shard.max_over_ranks(ms)
        q.put((rank, got, shard.shard_seeds(0, rank, 3)))
    finally:
        dist.destroy_process_group()


def test_max_over_ranks_gloo_world2():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    res = dict((r, (v, s)) for r, v, s in out)
    assert res[0][0] == res[1][0] == 150.0
    assert res[0][1] + res[1][1] == [i for i in range(6)]
