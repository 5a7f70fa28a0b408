"""Leaving a broken ``torch.distributed`` world and joining a new one.

Two ways to go on after a loss in the reference tier:

* at constant world size (a replacement takes the dead rank's place): every survivor leaves the
  default group that includes the dead rank (``leave_world``: abort on NCCL so nothing waits on the
  dead member, then destroy) and joins a fresh rendezvous with the replacement (``join_world``); the
  engine's own groups are rebuilt on top;
* smaller (SHRINK): the survivors' group from the old one (``shrink_world``, a
  :class:`~everserve_b200.runtime.shrink.ShrinkableGroup`).

A step of ``leave_world`` that fails is recorded, not raised: a rank that cannot leave cleanly must
still be able to join.

Reference parity: core/everserve/reference/world.py:21-57 (leave_world, join_world).
"""

from __future__ import annotations

import datetime

import torch.distributed as dist

from ..runtime.shrink import ShrinkableGroup


def leave_world() -> list[str]:
    """Abort (NCCL) and destroy the default process group with its subgroups; the steps that ran,
    for the event log ("abort", "destroy", or what failed)."""
    steps: list[str] = []
    if not dist.is_initialized():
        return steps
    try:
        if dist.get_backend() == "nccl":
            from torch.distributed import distributed_c10d as c10d

            c10d._abort_process_group()
            steps.append("abort")
    except Exception as e:  # noqa: BLE001 - recorded for the event log
        steps.append(f"abort failed: {type(e).__name__}: {e}")
    try:
        dist.destroy_process_group()
        steps.append("destroy")
    except Exception as e:  # noqa: BLE001 - recorded for the event log
        steps.append(f"destroy failed: {type(e).__name__}: {e}")
    return steps


def join_world(init_method: str, rank: int, world: int, backend: str = "gloo",
               timeout: datetime.timedelta = datetime.timedelta(seconds=120)) -> None:
    """Join a new default process group as `rank` of `world` at `init_method` (a rendezvous no
    earlier world used: a new epoch's address or store prefix)."""
    dist.init_process_group(backend, init_method=init_method, rank=rank, world_size=world, timeout=timeout)


def form_group(store, members: list[int], me: int, epoch: int = 0, timeout_s: float = 30.0,
               backend: str = "gloo") -> ShrinkableGroup:
    """A group of `members` over `store` (keyed by epoch), which the survivors can shrink."""
    return ShrinkableGroup(store, members, me, backend=backend, timeout_s=timeout_s, epoch=epoch)


def shrink_world(group: ShrinkableGroup, lost: list[int], epoch: int) -> ShrinkableGroup:
    """The survivors' group (every survivor calls it with the same `lost` and `epoch`)."""
    group.shrink(lost, epoch)
    return group
