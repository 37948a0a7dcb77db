"""The two collectives the tensor-parallel and page-split paths use.

With NCCL (one process per GPU, the serving and benchmark setup) they are plain
torch.distributed calls on the GPU tensors. A gloo group (ranks sharing one GPU,
as the one-GPU tests run the two-rank model) cannot take every collective on CUDA
tensors, so there the data is staged through host memory; the result is the same.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def _staged(x: torch.Tensor, group) -> bool:
    return x.is_cuda and dist.get_backend(group) == "gloo"


def all_reduce_(x: torch.Tensor, group=None) -> torch.Tensor:
    """In-place sum over the group."""
    if _staged(x, group):
        h = x.cpu()
        dist.all_reduce(h, group=group)
        x.copy_(h)
    else:
        dist.all_reduce(x, group=group)
    return x


def all_gather_into_(out: torch.Tensor, x: torch.Tensor, group=None) -> torch.Tensor:
    """out = the ranks' x one after the other (rank order)."""
    if _staged(x, group):
        h = torch.empty(out.numel(), dtype=out.dtype)
        dist.all_gather_into_tensor(h, x.cpu(), group=group)
        out.copy_(h.view_as(out))
    else:
        dist.all_gather_into_tensor(out, x, group=group)
    return out
