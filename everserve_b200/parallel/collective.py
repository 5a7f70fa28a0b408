"""The tensor-parallel collective the model's row-parallel layers go through.

``make_tp_collective`` builds the collective for one rank of the default process group: the
failure-detecting peer-memory kernels (fused GEMM + all-reduce) when ``kind == "fused"``, or the
plain NCCL path.
"""

from __future__ import annotations

import os

import torch

from .nccl import GroupCollective


def make_tp_collective(device: torch.device, kind: str = "fused", group=None):
    """kind: "fused" (NVLS multicast pushes when the node has them, else P2P), "p2p" (peer stores
    only: the variant for groups whose members may die), or "nccl"."""
    if kind in ("fused", "p2p"):
        from .fused import FusedTPCollective

        import torch.distributed as dist

        size = dist.get_world_size(group)
        if kind == "fused" and size >= 4 and os.environ.get("ES_NVLS", "1") != "0":
            try:
                return FusedTPCollective(device, group, nvls=True)
            except (RuntimeError, AttributeError, ImportError):
                pass
        return FusedTPCollective(device, group)
    return GroupCollective(group)
