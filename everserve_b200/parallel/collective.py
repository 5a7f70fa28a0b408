"""The tensor-parallel collective the model's row-parallel layers go through.

``make_tp_collective`` builds the collective for one rank of the default process group: the
failure-detecting peer-memory kernels (fused GEMM + all-reduce) when ``kind == "fused"``, or the
plain NCCL path.
"""

from __future__ import annotations

import torch

from .nccl import GroupCollective


def make_tp_collective(device: torch.device, kind: str = "fused", group=None):
    if kind == "fused":
        try:
            from .fused import FusedTPCollective
        except ImportError:
            FusedTPCollective = None  # noqa: N806
        if FusedTPCollective is not None:
            return FusedTPCollective(device, group)
    return GroupCollective(group)
