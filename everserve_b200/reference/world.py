"""Leaving and re-forming the reference tier's process group after a loss.

Reference parity: core/everserve/reference/world.py:21-57 (leave_world, join_world), over this
framework's ShrinkableGroup.
"""

from __future__ import annotations

from ..runtime.shrink import ShrinkableGroup


def join_world(store, members: list[int], me: int, epoch: int = 0, timeout_s: float = 30.0) -> ShrinkableGroup:
    return ShrinkableGroup(store, members, me, backend="gloo", timeout_s=timeout_s, epoch=epoch)


def leave_world(group: ShrinkableGroup, lost: list[int], epoch: int) -> ShrinkableGroup:
    """The survivors' group (every survivor calls it with the same `lost` and `epoch`)."""
    group.shrink(lost, epoch)
    return group
