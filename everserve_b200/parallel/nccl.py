"""Collectives over a torch.distributed process group (NCCL on GPUs, gloo on CPU).

This is the plain library path: the fallback for tensors the failure-detecting kernels do not
take, the pipeline transport, and the baseline the fused kernels are measured against.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


class GroupCollective:
    """all_reduce / all_gather / broadcast over one process group."""

    def __init__(self, group=None, ranks: list[int] | None = None):
        self.group = group
        self.ranks = ranks
        self.size = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0

    def all_reduce(self, t: torch.Tensor) -> torch.Tensor:
        if self.size > 1:
            dist.all_reduce(t, group=self.group)
        return t

    def all_gather(self, t: torch.Tensor) -> torch.Tensor:
        """Concatenate every rank's tensor along the last dim, in rank order."""
        if self.size == 1:
            return t
        parts = [torch.empty_like(t) for _ in range(self.size)]
        dist.all_gather(parts, t.contiguous(), group=self.group)
        return torch.cat(parts, dim=-1)

    def broadcast(self, t: torch.Tensor, src: int = 0) -> torch.Tensor:
        if self.size > 1:
            dist.broadcast(t, src=src if self.ranks is None else self.ranks[src], group=self.group)
        return t

    def barrier(self) -> None:
        if self.size > 1:
            dist.barrier(group=self.group)
