"""The order in which a process that took a position captures its CUDA graphs again.

Batch buckets are captured from the one the engine runs now outwards (its running batch first,
then the nearest larger and smaller ones), so the first steps after a change replay graphs while
the rest are captured beside them.

Reference parity: core/everserve/reference/recapture.py:20-45.
"""

from __future__ import annotations

from typing import Sequence


def next_slice(buckets: Sequence[int], done: set, running: int) -> int | None:
    """The next bucket to capture, or None when every bucket is done."""
    todo = [b for b in buckets if b not in done]
    if not todo:
        return None
    return min(todo, key=lambda b: (0 if b >= running else 1, abs(b - running), b))
