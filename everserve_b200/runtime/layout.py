"""Positions of an engine's ranks over its parallel dimensions, and the members of each group.

A member is a rank position (an ``int``) or a spare standing in for one (``"R<rank>"``). With data
and context parallel 1, rank ``r`` sits at pipeline stage ``r // tp`` and tensor column
``r % tp``: its tensor-parallel collectives run over the members of its stage, its pipeline sends
and receives over the members of its column. A collective's scope says whether it stays inside a
domain (one node's NVLink: the peer-memory kernels apply) or crosses the fabric (a library group).

Reference parity: the mapping rule and the ``R<rank>`` spare id of
core/everserve/comm/layout.py:1-80 and core/everserve/comm/shadow.py (the same rule, so a layout
and a member set mean the same positions on both sides of the wire).
"""

from __future__ import annotations

import enum
from dataclasses import dataclass
from typing import Sequence, Union

Member = Union[int, str]


class Scope(enum.Enum):
    DOMAIN = "domain"
    FABRIC = "fabric"


def is_replacement(m: Member) -> bool:
    return isinstance(m, str) and m.startswith("R")


def replacement(rank: int) -> str:
    return f"R{rank}"


def position(m: Member) -> int:
    """The rank position a member holds: its rank, or the rank a spare stands in for."""
    return int(m[1:]) if is_replacement(m) else int(m)


@dataclass(frozen=True)
class ParallelLayout:
    tensor_parallel: int = 1
    pipeline_parallel: int = 1
    data_parallel: int = 1
    expert_parallel: int = 1

    def __post_init__(self):
        if min(self.tensor_parallel, self.pipeline_parallel, self.data_parallel, self.expert_parallel) < 1:
            raise ValueError(f"every parallel size must be at least 1: {self}")

    @property
    def world(self) -> int:
        return self.tensor_parallel * self.pipeline_parallel * self.data_parallel

    def stage(self, m: Member) -> int:
        return (position(m) % (self.tensor_parallel * self.pipeline_parallel)) // self.tensor_parallel

    def column(self, m: Member) -> int:
        return position(m) % self.tensor_parallel

    def replica(self, m: Member) -> int:
        return position(m) // (self.tensor_parallel * self.pipeline_parallel)

    def tensor_members(self, members: Sequence[Member], me: Member) -> tuple[Member, ...]:
        s, d = self.stage(me), self.replica(me)
        return tuple(m for m in members if self.stage(m) == s and self.replica(m) == d)

    def pipeline_members(self, members: Sequence[Member], me: Member) -> tuple[Member, ...]:
        c, d = self.column(me), self.replica(me)
        return tuple(m for m in members if self.column(m) == c and self.replica(m) == d)

    def members_of(self, scope: Scope, members: Sequence[Member], me: Member) -> tuple[Member, ...]:
        return self.tensor_members(members, me) if scope is Scope.DOMAIN else self.pipeline_members(members, me)

    def next_stage(self, m: Member) -> int | None:
        """Rank position that receives this member's stage output (None on the last stage)."""
        s = self.stage(m)
        if s + 1 >= self.pipeline_parallel:
            return None
        return position(m) + self.tensor_parallel

    def prev_stage(self, m: Member) -> int | None:
        s = self.stage(m)
        if s == 0:
            return None
        return position(m) - self.tensor_parallel

    def last_stage_ranks(self) -> list[int]:
        base = (self.pipeline_parallel - 1) * self.tensor_parallel
        return [d * self.tensor_parallel * self.pipeline_parallel + base + c
                for d in range(self.data_parallel) for c in range(self.tensor_parallel)]
