"""Data-parallel host logic on CPU with two gloo ranks: every rank adopts rank 0's conv shift (rank 0 holds
global image 0, whose sums fix the shift in the reference), batches shard contiguously, and the stack's
column-parallel head (all-gather of hidden rows, then a vocabulary slice per rank) reassembles the full
logits."""

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
        # column-parallel head: rows of this rank's sequences -> all rows -> this rank's vocabulary slice
        h_local = torch.arange(2 * 4, dtype=torch.float32).view(2, 4) + 100 * rank
        h_all = torch.empty(2 * world, 4)
        parallel.gather_rows(h_local, h_all)
        w = torch.arange(6 * 4, dtype=torch.float32).view(6, 4)
        n_cols = 6 // world
        logits = h_all @ w[rank * n_cols:(rank + 1) * n_cols].t()
        q.put((rank, own, s1, s2, part[:, 0].tolist(), h_all.tolist(), logits.tolist()))
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
    assert res[0][:5] == (0, 10, 10, 20, [0, 3, 6, 9])
    assert res[1][:5] == (1, 11, 10, 20, [12, 15, 18, 21])
    h_all = torch.tensor(res[0][5])
    want_h = torch.cat([torch.arange(8, dtype=torch.float32).view(2, 4) + 100 * r for r in range(2)])
    assert torch.equal(h_all, want_h) and res[1][5] == res[0][5]
    w = torch.arange(6 * 4, dtype=torch.float32).view(6, 4)
    logits = torch.cat([torch.tensor(res[r][6]) for r in range(2)], dim=1)
    assert torch.equal(logits, want_h @ w.t())


def test_shard_rejects_uneven():
    from torch_xdna import parallel

    with pytest.raises(ValueError):
        parallel.shard(torch.zeros(5), 0, 2)
