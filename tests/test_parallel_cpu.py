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


def _strip_worker(rank, world, port, q):
    """One rank of an image split into strips of rows: the per-image max and the calibration max combined
    over ranks, the strip quantised with the combined scale into the bordered layout, the halo rows
    exchanged, and the strip's exact conv sums read off its bordered rows -- compared with the whole image."""
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "torch-xdna_b200"))
    sys.path.insert(0, root)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import numpy as np

        from oracle import xdna_oracle as orc
        from torch_xdna import parallel

        g = np.random.default_rng(17)
        N, C, Co, H, W = 2, 5, 4, 11, 7
        x = g.standard_normal((N, C, H, W)).astype(np.float32)
        wq = g.integers(-127, 128, (Co, C, 3, 3)).astype(np.int8)
        r0, r1 = parallel.strip_rows(H, rank, world)
        rows = r1 - r0
        xl = x[:, :, r0:r1]
        # per-image max |x| as bit patterns, combined over the strips
        amax = torch.from_numpy(np.abs(xl).reshape(N, -1).max(axis=1).astype(np.float32).view(np.int32).copy())
        parallel.all_max_(amax)
        xq_all, s_all = orc.conv_quant(x)
        ok_amax = np.array_equal(amax.numpy().view(np.float32), np.abs(x).reshape(N, -1).max(axis=1))
        s = (np.maximum(amax.numpy().view(np.float32), np.float32(1e-8)) / np.float32(127)).astype(np.float32)
        # this strip quantised into the bordered NHWC layout, border rows zero, then the halo
        xp = torch.zeros(N, rows + 2, W + 2, C, dtype=torch.int8)
        xp[:, 1:rows + 1, 1:W + 1] = torch.from_numpy(
            np.clip(np.rint(xl / s[:, None, None, None]), -127, 127).astype(np.int8)).permute(0, 2, 3, 1)
        parallel.exchange_halo(xp)
        # the strip's sums: the 3x3 conv over its bordered rows with no further padding
        acc = torch.nn.functional.conv2d(xp.permute(0, 3, 1, 2).double(), torch.from_numpy(wq).double()).to(torch.int32)
        want = orc.conv_acc(xq_all, wq)[:, :, r0:r1]
        ok_acc = np.array_equal(acc.numpy(), want)
        # the calibration max of image 0's sums, combined over the strips
        top = torch.tensor([int(acc[0].abs().max())], dtype=torch.int32)
        parallel.all_max_(top)
        ok_top = int(top) == int(np.abs(orc.conv_acc(xq_all, wq)[0]).max())
        q.put((rank, (r0, r1), ok_amax, bool(np.array_equal(s, s_all)), ok_acc, ok_top))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_image_strips_halo_and_combined_maxima(world):
    """Image strips for batch-1 convs: 11 rows over 2 or 3 ranks (the middle rank exchanges both halos)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_strip_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=10) for _ in range(world))
    spans = [r[1] for r in res]
    assert spans[0][0] == 0 and spans[-1][1] == 11 and all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    for r in res:
        assert r[2:] == (True, True, True, True), r


def _dead_peer_worker(rank, world, port, q):
    """Rank 1 leaves (raises) between steps, before the strip exchange; rank 0's next collective must end
    with an error within the process group's timeout instead of waiting for good."""
    import datetime
    import sys
    import time

    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "torch-xdna_b200"))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    from torch_xdna import parallel

    top = torch.tensor([5 + rank], dtype=torch.int32)
    parallel.all_max_(top)  # a step both ranks complete
    if rank == 1:
        q.put((1, int(top), "left"))
        raise SystemExit(3)  # the failure, on the host: this rank never joins the next exchange
    t0 = time.monotonic()
    xp = torch.zeros(1, 4, 6, 16, dtype=torch.int8)
    try:
        parallel.exchange_halo(xp)
        outcome = "completed"
    except Exception as e:  # the timeout surfaces as a RuntimeError from the backend
        outcome = type(e).__name__
    q.put((0, int(top), outcome, time.monotonic() - t0))


def test_dead_peer_ends_the_exchange_with_an_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dead_peer_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    res = sorted(q.get(timeout=10) for _ in range(2))
    assert procs[1].exitcode == 3
    assert res[0][1] == res[1][1] == 6          # the step before the failure completed on both ranks
    assert res[0][2] != "completed" and res[0][3] < 60, res[0]


def test_shard_rejects_uneven():
    from torch_xdna import parallel

    with pytest.raises(ValueError):
        parallel.shard(torch.zeros(5), 0, 2)
