"""Tensor-parallel decode across the GPUs of one box: one process per GPU.

    import torch.distributed as dist
    dist.init_process_group("nccl", ...)          # or "gloo": only bytes travel
    m = fwb.tp.open_model(path, max_ctx, rank, world, device)

The only host-side exchange is the 64-byte CUDA IPC handle of every rank's
exchange buffer (all_gather_object over the process group).  From then on
the ranks meet only on the GPUs: the partial sums after o-proj and down-proj
and the greedy-token candidates are read over NVLink inside the persistent
decode kernel.  Every rank must make the same forward calls with the same
tokens and positions.
"""
from __future__ import annotations

from .model import Model


def gather_handles(handle: bytes, group=None) -> list[bytes]:
    """All-gather one bytes object per rank, returned in rank order."""
    import torch.distributed as dist

    out: list = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, handle, group=group)
    return [bytes(x) for x in out]


def open_model(path: str, max_ctx: int, rank: int, world: int, device: int, group=None) -> Model:
    return Model(path, max_ctx=max_ctx, device=device, rank=rank, world=world,
                 exchange=lambda h: gather_handles(h, group))
