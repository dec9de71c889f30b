"""The N > 1 path of bench.py on CPU: two gloo ranks shard the decisions with
no overlap and agree on the slowest rank's time (the max-over-ranks rule)."""

import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        import bench
        batches = bench.make_batches(rank, 2, 4, 152064, 20261201)
        ids = [b.input_ids[:b.rows[0].real_len].tolist() for b in batches]
        my_ms = 100.0 * (rank + 1)          # rank 1 is the slow one
        slow = bench.max_over_ranks(my_ms, world)
        out[rank] = (ids, slow, bench.whole_job_rate(8, world, slow))
    finally:
        dist.destroy_process_group()


def test_two_ranks_shard_and_take_the_slowest_time():
    world, port = 2, _free_port()
    out = mp.Manager().dict()
    mp.spawn(_rank, args=(world, port, out), nprocs=world, join=True)
    ids0, slow0, rate0 = out[0]
    ids1, slow1, rate1 = out[1]
    assert slow0 == slow1 == 200.0
    assert rate0 == rate1 == pytest.approx(8 * 2 / 0.2)
    assert not any(a == b for a in ids0 for b in ids1)  # no decision on two ranks
