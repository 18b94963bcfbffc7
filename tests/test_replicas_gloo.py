"""Multi-process (one rank per GPU) logic on CPU: two gloo ranks on 127.0.0.1.

The data-parallel path has no data collective; what spans ranks is the image
split and the end-of-run reduction (max of device times, sum of images) that
bench.py reports as whole-job throughput."""
import os
import socket

import pytest
import torch.multiprocessing as mp

from pdefa_b200.replicas import job_throughput, shard_bounds


def test_shard_bounds_cover_every_image_once():
    for n in (0, 1, 7, 256, 257, 1000):
        for world in (1, 2, 3, 8):
            seen = []
            for r in range(world):
                lo, hi = shard_bounds(n, r, world)
                assert 0 <= lo <= hi <= n
                seen.extend(range(lo, hi))
            assert seen == list(range(n))
    with pytest.raises(ValueError):
        shard_bounds(4, 2, 2)


def test_job_throughput():
    assert job_throughput(512, 1000.0) == 512.0
    with pytest.raises(ValueError):
        job_throughput(1, 0.0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out):
    import datetime

    import torch.distributed as dist

    from pdefa_b200.replicas import reduce_job, shard_bounds

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        lo, hi = shard_bounds(10, rank, world)
        # rank r "took" 3 + r ms for its shard
        out[rank] = (lo, hi) + reduce_job(3.0 + rank, hi - lo)
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_reduce_max_time_and_total_images():
    world = 2
    port = _free_port()
    with mp.get_context("spawn").Manager() as m:
        out = m.dict()
        mp.spawn(_rank_main, args=(world, port, out), nprocs=world, join=True)
        res = dict(out)
    assert res[0][:2] == (0, 5) and res[1][:2] == (5, 10)
    for r in range(world):
        assert res[r][2] == 4.0          # slowest rank's time on every rank
        assert res[r][3] == 10           # every image counted once
    assert job_throughput(res[0][3], res[0][2]) == 2500.0
