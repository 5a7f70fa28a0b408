"""What happens when a rank leaves: one enum shared by the runtime, the policy and the engine.

Reference parity: core/everserve/outcome.py:13-21 (the same three outcomes and their wire values in
``signals.Outcome``).
"""

from __future__ import annotations

import enum

from .proto import signals as sp


class Outcome(str, enum.Enum):
    REPLACE = "replace"  # a spare takes the lost rank's position at constant world size
    SHRINK = "shrink"  # the survivors absorb the lost rank's units (placement-independent model)
    REBUILD = "rebuild"  # the engine restarts at a smaller size and replays its requests

    @property
    def wire(self) -> int:
        return {Outcome.REPLACE: sp.OUTCOME_REPLACE, Outcome.SHRINK: sp.OUTCOME_SHRINK,
                Outcome.REBUILD: sp.OUTCOME_REBUILD}[self]

    @classmethod
    def from_wire(cls, v: int) -> "Outcome":
        return {sp.OUTCOME_REPLACE: cls.REPLACE, sp.OUTCOME_SHRINK: cls.SHRINK, sp.OUTCOME_REBUILD: cls.REBUILD}[v]
