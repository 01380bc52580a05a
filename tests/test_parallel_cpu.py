"""Data-parallel host logic on CPU with two gloo ranks: every rank adopts rank 0's conv shift (rank 0 holds
global image 0, whose sums fix the shift in the reference), and batches shard contiguously."""

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


def _worker(rank, world, port, q):
    import sys

    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "torch-xdna_b200"))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from torch_xdna import parallel

        # before enabling: each rank keeps its own shift
        own = parallel.broadcast_shift(10 + rank, "cpu")
        parallel.enable_data_parallel()
        # two layers calibrated in the same order on every rank: rank 0's shifts win
        s1 = parallel.broadcast_shift(10 + rank, "cpu")
        s2 = parallel.broadcast_shift(20 + 3 * rank, "cpu")
        parallel.disable_data_parallel()
        x = torch.arange(8 * 3).view(8, 3)
        part = parallel.shard(x, rank, world)
        q.put((rank, own, s1, s2, part[:, 0].tolist()))
    finally:
        dist.destroy_process_group()


def test_shift_broadcast_and_shards_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=10) for _ in range(2))
    assert res[0] == (0, 10, 10, 20, [0, 3, 6, 9])
    assert res[1] == (1, 11, 10, 20, [12, 15, 18, 21])


def test_shard_rejects_uneven():
    from torch_xdna import parallel

    with pytest.raises(ValueError):
        parallel.shard(torch.zeros(5), 0, 2)
