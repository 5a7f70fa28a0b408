"""Staging a departing rank's KV in rounds before its notice runs out.

``blocks_to_stage(blocks, per_round)`` orders the blocks a departing rank must hand over, oldest
write first (the newest blocks are still being written until the rank leaves; the spare catches
up on those at the boundary), and splits them into rounds of at most `per_round` blocks each.

Reference parity: core/everserve/reference/staging.py:25-94.
"""

from __future__ import annotations

from typing import Sequence


def blocks_to_stage(blocks: Sequence[tuple[int, int]], per_round: int) -> list[list[int]]:
    """`blocks`: (block id, step last written). Rounds of block ids, oldest writes first."""
    if per_round <= 0:
        raise ValueError("per_round must be positive")
    order = [b for b, _ in sorted(blocks, key=lambda x: (x[1], x[0]))]
    return [order[i : i + per_round] for i in range(0, len(order), per_round)]
