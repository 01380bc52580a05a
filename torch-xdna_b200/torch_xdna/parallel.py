"""Data parallelism across the GPUs of one box: one process per GPU, torch.distributed over NCCL.

What shards (the reference is single-device; the build adds these):
  - conv batches: images are independent (each has its own activation scale), so a batch splits over
    ranks with no exchange -- except the requantise shift, which the reference fixes from the first
    image of the first call (R:torch_xdna/conv.py:171-172). With enable_data_parallel(), every conv
    layer's first calibration takes the shift computed on rank 0 (which holds global image 0) and
    broadcasts it, so every rank requantises exactly as one GPU running the whole batch would;
  - stack sequences: sequences are independent under the mask, so the layers split over ranks with no
    collective at all; the linear head can then run column-parallel (each rank 1/world of the
    vocabulary for every token) after gather_rows of the final hidden states;
  - the W8A8 linears do not shard usefully (their outputs are larger than their work): replicas.
"""

import torch

_state = {"group": None, "enabled": False}


def enable_data_parallel(group=None):
    """Conv calibrations from now on use rank 0's shift (torch.distributed must be initialised)."""
    import torch.distributed as dist

    if not dist.is_initialized():
        raise RuntimeError("enable_data_parallel needs torch.distributed.init_process_group first")
    _state["group"], _state["enabled"] = group, True


def disable_data_parallel():
    _state["group"], _state["enabled"] = None, False


def enabled() -> bool:
    return _state["enabled"]


def broadcast_shift(shift: int, device) -> int:
    """The shift every rank must use: rank 0's. Every rank calls this for the same layers in the same order
    (the first call of each conv layer), so the broadcasts pair up."""
    if not _state["enabled"]:
        return shift
    import torch.distributed as dist

    group = _state["group"]
    src = dist.get_global_rank(group, 0) if group is not None else 0
    t = torch.tensor([shift], dtype=torch.int32, device=device)
    dist.broadcast(t, src=src, group=group)
    return int(t.item())


def strip_rows(H: int, rank: int, world: int):
    """Rows [r0, r1) of an H-row image that rank `rank` of `world` holds: equal strips, the first H % world
    ranks one row more."""
    base, extra = divmod(H, world)
    r0 = rank * base + min(rank, extra)
    return r0, r0 + base + (1 if rank < extra else 0)


def all_max_(t: torch.Tensor, group=None) -> torch.Tensor:
    """t = the elementwise max of t over the ranks (in place). Non-negative float bit patterns held as int32
    (per-image maxima of |x|) order like their values, so their max is the max of the values, bit for bit."""
    import torch.distributed as dist

    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return t


def exchange_halo(xp: torch.Tensor, group=None) -> torch.Tensor:
    """The 1-row halo of a strip in the bordered layout xp [N, rows + 2, W + 2, Cp] (rows 1..rows this rank's
    own): row 0 receives the last own row of the rank above, row rows + 1 the first own row of the rank below;
    the image's top and bottom ranks keep their zero border. Every rank calls it in the same order."""
    import torch.distributed as dist

    rank, world = dist.get_rank(group), dist.get_world_size(group)
    if world == 1:
        return xp
    peer = (lambda r: dist.get_global_rank(group, r)) if group is not None else (lambda r: r)
    rows = xp.shape[1] - 2
    send_up, send_dn = xp[:, 1].contiguous(), xp[:, rows].contiguous()
    recv_up, recv_dn = torch.empty_like(send_up), torch.empty_like(send_dn)
    ops = []
    if rank > 0:
        ops += [dist.P2POp(dist.isend, send_up, peer(rank - 1), group), dist.P2POp(dist.irecv, recv_up, peer(rank - 1), group)]
    if rank < world - 1:
        ops += [dist.P2POp(dist.isend, send_dn, peer(rank + 1), group), dist.P2POp(dist.irecv, recv_dn, peer(rank + 1), group)]
    for req in dist.batch_isend_irecv(ops):
        req.wait()
    if rank > 0:
        xp[:, 0] = recv_up
    if rank < world - 1:
        xp[:, rows + 1] = recv_dn
    return xp


def shard(t: torch.Tensor, rank: int, world: int, dim: int = 0) -> torch.Tensor:
    """This rank's contiguous slice of `t` along `dim` (rank 0 holds the first elements)."""
    n = t.shape[dim]
    if n % world:
        raise ValueError(f"{n} items do not divide over {world} ranks")
    k = n // world
    return t.narrow(dim, rank * k, k)


def gather_rows(local: torch.Tensor, out: torch.Tensor, group=None) -> torch.Tensor:
    """out [world x rows, ...] = every rank's `local` [rows, ...] in rank order (an NCCL all-gather over
    NVLink on GPUs): the hidden states of all sequences for a column-parallel head."""
    import torch.distributed as dist

    assert out.shape[0] == local.shape[0] * dist.get_world_size(group) and out.shape[1:] == local.shape[1:]
    dist.all_gather_into_tensor(out, local.contiguous(), group=group)
    return out


class RowGather:
    """Every rank's [rows, cols] bf16 buffer as the row-concatenated A operand of the column-parallel head
    GEMM, gathered and multiplied in one pipeline instead of an all-gather followed by a GEMM.

    Each rank's buffer is a shareable allocation whose peers map it through CUDA IPC (NVLink). gemm():
      - "pipelined" (default): the GEMM over this rank's own rows starts at once; meanwhile a copy engine
        brings every peer's block across NVLink exactly once, in ring order, into local staging, and the
        GEMM over each peer's rows starts as soon as its block has landed (copies overlap the math);
      - "direct": one GEMM whose TMA producer reads the peers' rows straight from their memory
        (xdna_gemm_bf16_gather). Every column tile re-reads its A rows, and remote rows do not stay in
        this GPU's L2, so each remote row crosses NVLink once per column tile: correct, but slower.
    `local` is this rank's buffer; write it, then call gemm() on every rank in the same order (it brackets
    the work with two one-element all-reduces, the device-side barriers that order every rank's writes of
    `local` before the peers read it, and the reads before the next writes)."""

    def __init__(self, rows: int, cols: int, device, group=None, mode: str = "pipelined"):
        import torch.distributed as dist

        from . import kernels

        assert mode in ("pipelined", "direct")
        self.group, self.mode = group, mode
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.rows, self.cols = rows, cols
        self.local, self._ptr = kernels.ipc_alloc((rows, cols), device)
        mine = torch.frombuffer(bytearray(kernels.ipc_handle(self._ptr)), dtype=torch.uint8).to(device)
        everyone = torch.empty(self.world * 64, dtype=torch.uint8, device=device)
        dist.all_gather_into_tensor(everyone, mine, group=group)
        handles = everyone.cpu().numpy().tobytes()
        self.ptrs = [self._ptr if r == self.rank else kernels.ipc_open(handles[64 * r:64 * (r + 1)])
                     for r in range(self.world)]
        self.peers = [kernels.device_view(p, (rows, cols), device) if r != self.rank else self.local
                      for r, p in enumerate(self.ptrs)]
        self.staged = {r: torch.empty(rows, cols, dtype=torch.bfloat16, device=device)
                       for r in range(self.world) if r != self.rank} if mode == "pipelined" else {}
        self.maps = torch.empty(self.world * 128, dtype=torch.uint8, device=device)   # allocator blocks: 512-aligned
        self._copy = torch.cuda.Stream(device)
        self._landed = {r: torch.cuda.Event() for r in self.staged}
        self._flag = torch.zeros(1, device=device)

    def gemm(self, w: torch.Tensor, out: torch.Tensor, bias=None) -> torch.Tensor:
        """out [world * rows, N] = (all ranks' `local`, in rank order) . w^T, w [N, cols]."""
        import torch.distributed as dist

        from . import kernels

        dist.all_reduce(self._flag, group=self.group)        # every rank's `local` is written
        if self.mode == "direct":
            kernels.gemm_bf16_gather(self.ptrs, self.rows, self.cols, w, out, self.maps, bias)
        else:
            cur = torch.cuda.current_stream()
            self._copy.wait_stream(cur)
            with torch.cuda.stream(self._copy):              # every peer block crosses NVLink once
                for k in range(1, self.world):
                    r = (self.rank + k) % self.world
                    self.staged[r].copy_(self.peers[r], non_blocking=True)
                    self._landed[r].record(self._copy)
            rows = self.rows
            kernels.gemm_bf16(self.local, w, kernels.GEMM_F32ACC, out=out[self.rank * rows:(self.rank + 1) * rows],
                              bias=bias)
            for k in range(1, self.world):
                r = (self.rank + k) % self.world
                cur.wait_event(self._landed[r])
                kernels.gemm_bf16(self.staged[r], w, kernels.GEMM_F32ACC, out=out[r * rows:(r + 1) * rows],
                                  bias=bias)
        dist.all_reduce(self._flag, group=self.group)        # every rank has read them
        return out

    def exchange(self):
        """The exchange of gemm() without the GEMMs ("pipelined" mode): every peer block copied over NVLink
        into local staging, bracketed by the same two flag all-reduces, the current stream waiting for the
        copies. Measures the NVLink share of the pipelined head."""
        import torch.distributed as dist

        assert self.mode == "pipelined"
        dist.all_reduce(self._flag, group=self.group)
        cur = torch.cuda.current_stream()
        self._copy.wait_stream(cur)
        with torch.cuda.stream(self._copy):
            for k in range(1, self.world):
                r = (self.rank + k) % self.world
                self.staged[r].copy_(self.peers[r], non_blocking=True)
        cur.wait_stream(self._copy)
        dist.all_reduce(self._flag, group=self.group)

    def close(self):
        import torch.distributed as dist

        from . import kernels

        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        self.peers = None
        for r, p in enumerate(self.ptrs):
            if r != self.rank:
                kernels.ipc_close(p)
        dist.barrier(group=self.group)                       # no peer still maps `local`
        self.local = None
        kernels.ipc_free(self._ptr)
