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
