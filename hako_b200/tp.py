"""Tensor-parallel group setup over a torch.distributed process group (or any
transport that can all-gather bytes): every rank exports its context's
exchange handle, all ranks gather all handles in rank order and connect.
torch.distributed is plumbing here only; the data path is the step kernel's
peer stores."""
from __future__ import annotations


def all_gather_bytes(data: bytes, pg=None) -> list:
    """All ranks' `data` in rank order, over torch.distributed (default group
    unless `pg` is given); any backend (gloo, nccl)."""
    import torch.distributed as dist
    out = [None] * dist.get_world_size(pg)
    dist.all_gather_object(out, data, group=pg)
    return out


def connect(ctx, pg=None) -> None:
    """Join `ctx` (a HakmCtx on this rank's GPU) to the group of all ranks of
    the process group."""
    import torch.distributed as dist
    handles = all_gather_bytes(ctx.tp_export(), pg)
    ctx.tp_connect(dist.get_rank(pg), handles)
