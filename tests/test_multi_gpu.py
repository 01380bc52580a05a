"""The multi-GPU code paths on real GPUs, two NCCL ranks as child processes (skipped with fewer than 2 GPUs):

- parallel.RowGather, pipelined (peer blocks copied over NVLink into local staging while the GEMM over this
  rank's rows runs) and direct (the GEMM's TMA reading peer rows): the column-parallel head's logits equal
  one GEMM over every rank's rows, bit for bit;
- conv data parallelism: rank 1 adopts rank 0's calibrated shift (NCCL broadcast), so the sharded batch gives
  exactly the whole batch's output on one GPU;
- image strips (conv.conv3x3_strip): an image split into row strips over the ranks, with the image max and
  the calibration max all-reduced and 1-row halos exchanged, gives exactly the whole image's output.
"""

import os
import socket

import pytest
import torch

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                                 reason="needs 2 GPUs")]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    import datetime
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "torch-xdna_b200"))
    sys.path.insert(0, root)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    out = {"rank": rank}
    try:
        import torch_xdna
        from torch_xdna import conv as xconv
        from torch_xdna import kernels, parallel

        with torch.no_grad():
            # ---- the column-parallel head: every rank's hidden rows x this rank's vocabulary slice
            rows, N = 512, 2048
            g = torch.Generator(device=dev).manual_seed(7)
            h_all = (torch.randn(world * rows, 1024, device=dev, generator=g)).to(torch.bfloat16)
            w_all = (torch.randn(N * world, 1024, device=dev, generator=g) * 0.03).to(torch.bfloat16)
            w = w_all[rank * N:(rank + 1) * N].contiguous()
            want = torch.empty(world * rows, N, dtype=torch.bfloat16, device=dev)
            kernels.gemm_bf16(h_all, w, kernels.GEMM_F32ACC, out=want)
            for mode in ("pipelined", "direct"):
                rg = parallel.RowGather(rows, 1024, dev, mode=mode)
                rg.local.copy_(h_all[rank * rows:(rank + 1) * rows])
                got = torch.empty_like(want)
                rg.gemm(w, got)
                torch.cuda.synchronize()
                out[f"head_{mode}"] = bool(torch.equal(got, want))
                rg.close()
            # ---- conv data parallelism: rank 0's shift broadcast
            cfg = torch_xdna.Config(verify="off")
            gw = torch.Generator(device=dev).manual_seed(3)
            wt = torch.randn(64, 32, 3, 3, device=dev, generator=gw) * 0.08
            x = torch.randn(4, 32, 20, 24, device=dev, generator=gw)
            x[0] *= 3.0      # image 0 (rank 0's) sets the shift; rank 1's images alone would give another
            whole = xconv.conv3x3_fused(cfg, x, torch.nn.Parameter(wt.clone()), None, True)
            parallel.enable_data_parallel()
            part = xconv.conv3x3_fused(cfg, x[2 * rank:2 * rank + 2].contiguous(), torch.nn.Parameter(wt.clone()),
                                       None, True)
            parallel.disable_data_parallel()
            out["conv_dp"] = bool(torch.equal(part, whole[2 * rank:2 * rank + 2]))
            # ---- image strips: two convs over a 2 x 48 x 40 batch split into row strips
            ws = [torch.randn(48, 48, 3, 3, device=dev, generator=gw) * 0.07 for _ in range(2)]
            xi = torch.randn(2, 48, 37, 40, device=dev, generator=gw)
            r0, r1 = parallel.strip_rows(37, rank, world)
            h, ref = xi[:, :, r0:r1].contiguous(), xi
            for wi in ws:
                h = xconv.conv3x3_strip(cfg, h, torch.nn.Parameter(wi.clone()), None, True)
                ref = xconv.conv3x3_fused(cfg, ref, torch.nn.Parameter(wi.clone()), None, True)
            out["strips"] = bool(torch.equal(h, ref[:, :, r0:r1]))
            out["device_error"] = kernels.take_device_error()
    except Exception as e:  # reported to the parent, which fails the test
        out["error"] = f"{type(e).__name__}: {e}"
    finally:
        q.put(out)
        dist.destroy_process_group()


def test_multi_gpu_paths_two_ranks():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    for p in procs:
        if p.is_alive():
            p.kill()
    res = [q.get(timeout=10) for _ in range(2)]
    for r in res:
        assert "error" not in r, r
        assert r["head_pipelined"] and r["head_direct"], r
        assert r["conv_dp"], r
        assert r["strips"], r
        assert r["device_error"] == (0, 0), r
