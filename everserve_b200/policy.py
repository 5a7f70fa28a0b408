"""A typed view of the policy document (``everserve.policy.v1.Policy``, proto3 JSON on disk).

``load`` / ``from_bytes`` / ``from_message`` give a frozen :class:`Policy`; ``choose_outcome`` is the
first outcome in the policy's order whose precondition holds (REPLACE needs a ready spare, SHRINK a
placement-independent model, REBUILD nothing; a policy naming only impossible outcomes falls back
to REBUILD); ``sets_to_preform`` lists the member sets an engine forms ahead of a loss (every
survivor set under SHRINK, one replacement set per standing spare under REPLACE), in a fixed
order every process agrees on.

Reference parity: core/everserve/policy.py:45-342 (same fields, same rules; the coordinator's C++
copy of the outcome rule is cpp/coord/state.cpp).
"""

from __future__ import annotations

import enum
import itertools
from dataclasses import dataclass, field
from pathlib import Path
from typing import Sequence

from google.protobuf import json_format

from .outcome import Outcome
from .proto import policy as pp
from .runtime.layout import Member, replacement

NOTICE_TRANSIT_S = 0.5  # what a notice needs to reach every rank through the control plane


class Guarantee(str, enum.Enum):
    EXACT = "exact"  # outputs identical to a no-fault run (deterministic kernels, exact replay)
    CONTINUOUS = "continuous"  # streams continue; outputs may differ after a change


class Loading(str, enum.Enum):
    PRELOADED = "preloaded"
    ON_NOTICE = "on_notice"


@dataclass(frozen=True)
class PlacedMember:
    node: str
    device: int


@dataclass(frozen=True)
class SpareSlot:
    node: str
    device: int
    rank: int | None = None  # None: stands for any rank


@dataclass(frozen=True)
class SpareLaunch:
    command: tuple[str, ...]
    env: tuple[tuple[str, str], ...] = ()


@dataclass(frozen=True)
class Engine:
    name: str
    members: tuple[PlacedMember, ...] = ()
    tensor_parallel: int = 1
    expert_parallel: int = 1
    pipeline_parallel: int = 1
    placement_independent_model: bool = False
    data_parallel: int = 1
    head_on_demand: bool = False
    spare_nodes: tuple[str, ...] = ()
    replica_nodes: tuple[str, ...] = ()
    guarantee: Guarantee = Guarantee.EXACT
    fabric_collectives: bool = False
    spares: tuple[SpareSlot, ...] = ()
    spare_launch: SpareLaunch | None = None
    release_bound_ms: int | None = None

    @property
    def world_size(self) -> int:
        return self.tensor_parallel * self.pipeline_parallel * self.data_parallel

    @property
    def spare_ranks(self) -> tuple[int, ...]:
        return tuple(s.rank for s in self.spares if s.rank is not None)

    def spare_node(self, rank: int) -> str | None:
        return next((s.node for s in self.spares if s.rank == rank), None)


@dataclass(frozen=True)
class Policy:
    version: str = ""
    outcomes_in_order: tuple[Outcome, ...] = (Outcome.REPLACE,)
    spares_per_engine: int = 0
    spare_loading: Loading = Loading.PRELOADED
    max_concurrent_losses: int = 0
    notice_min_ms: int = 0
    engines: tuple[Engine, ...] = field(default_factory=tuple)
    cover_planned: bool = False
    cover_form_timeout_ms: int = 30_000
    cover_max_groups_per_gpu: int = 0

    def engine(self, name: str) -> Engine:
        for e in self.engines:
            if e.name == name:
                return e
        raise KeyError(f"the policy names no engine {name!r}")

    def notice_lead_s(self, wanted_s: float) -> float:
        """How early a departure must be noticed: the wanted lead, at least the policy's floor."""
        return max(wanted_s, self.notice_min_ms / 1000.0) + NOTICE_TRANSIT_S


def _engine(e) -> Engine:
    return Engine(
        name=e.name,
        members=tuple(PlacedMember(m.node, m.device) for m in e.members),
        tensor_parallel=max(1, e.tensor_parallel), expert_parallel=max(1, e.expert_parallel),
        pipeline_parallel=max(1, e.pipeline_parallel), data_parallel=max(1, e.data_parallel),
        placement_independent_model=e.placement_independent_model, head_on_demand=e.head_on_demand,
        spare_nodes=tuple(e.spare_nodes), replica_nodes=tuple(e.replica_nodes),
        guarantee=Guarantee.CONTINUOUS if e.guarantee == pp.GUARANTEE_CONTINUOUS else Guarantee.EXACT,
        fabric_collectives=e.fabric_collectives,
        spares=tuple(SpareSlot(s.node, s.device, s.rank if s.HasField("rank") else None) for s in e.spares),
        spare_launch=SpareLaunch(tuple(e.spare_launch.command), tuple(sorted(e.spare_launch.env.items())))
        if e.HasField("spare_launch") and e.spare_launch.command else None,
        release_bound_ms=e.release_bound_ms if e.HasField("release_bound_ms") else None)


def from_message(msg) -> Policy:
    outcomes = tuple(Outcome.from_wire(o) for o in msg.outcomes_in_order if o) or (Outcome.REPLACE,)
    names = [e.name for e in msg.engines]
    if len(set(names)) != len(names):
        raise ValueError("the policy names an engine twice")
    return Policy(
        version=msg.version, outcomes_in_order=outcomes, spares_per_engine=msg.spares.per_engine,
        spare_loading=Loading.ON_NOTICE if msg.spares.loading == pp.SparePool.LOADING_ON_NOTICE else Loading.PRELOADED,
        max_concurrent_losses=msg.max_concurrent_losses, notice_min_ms=msg.notice_min_ms,
        engines=tuple(_engine(e) for e in msg.engines), cover_planned=msg.cover.enabled,
        cover_form_timeout_ms=msg.cover.form_timeout_ms or 30_000,
        cover_max_groups_per_gpu=msg.cover.max_groups_per_gpu)


def from_json(text: str) -> Policy:
    return from_message(json_format.Parse(text, pp.Policy()))


def from_bytes(data: bytes) -> Policy:
    msg = pp.Policy()
    msg.ParseFromString(data)
    return from_message(msg)


def load(path: str | Path) -> Policy:
    return from_json(Path(path).read_text())


def choose_outcome(policy: Policy, *, spare_ready: bool, placement_independent_model: bool) -> Outcome:
    for o in policy.outcomes_in_order:
        if o is Outcome.REPLACE and spare_ready:
            return o
        if o is Outcome.SHRINK and placement_independent_model:
            return o
        if o is Outcome.REBUILD:
            return o
    return Outcome.REBUILD


def member_sets(world: int, losses: Sequence[Sequence[int]] | None = None,
                replacements: Sequence[Sequence[int]] = ()) -> list[tuple[Member, ...]]:
    """Member sets of a world of `world` ranks: each loss set removed (every single loss when
    `losses` is None), or each replacement set's ranks held by their spares (``R<rank>``)."""
    out = []
    if replacements:
        for reps in replacements:
            out.append(tuple(replacement(r) if r in reps else r for r in range(world)))
        return out
    for lost in (losses if losses is not None else [(r,) for r in range(world)]):
        out.append(tuple(r for r in range(world) if r not in lost))
    return out


def sets_to_preform(policy: Policy, engine: Engine, spare_ranks: Sequence[int] = ()) -> list[tuple[Member, ...]]:
    """The member sets an engine forms groups for before any loss, in one order every process
    derives alike: the survivor sets of each single loss when the policy can shrink, then, when it
    can replace, the set in which each standing spare holds its rank. Spares the policy could never
    use, or for ranks the engine does not have, are a configuration error."""
    world = engine.world_size
    standing = sorted({int(r) for r in spare_ranks})
    enabled = set(policy.outcomes_in_order)
    errors = []
    if standing and Outcome.REPLACE not in enabled:
        errors.append(f"standing spares {standing} would never be used: the policy has no REPLACE outcome")
    stray = [r for r in standing if r < 0 or r >= world]
    if stray:
        errors.append(f"standing spares name ranks {stray}, but the engine has ranks 0..{world - 1}")
    if errors:
        raise ValueError("; ".join(errors))
    planned: list[tuple[Member, ...]] = []
    if Outcome.SHRINK in enabled:
        planned += member_sets(world)
    if Outcome.REPLACE in enabled and standing:
        planned += member_sets(world, replacements=[(r,) for r in standing])
    return planned


def loss_sets(world: int, max_losses: int) -> list[tuple[int, ...]]:
    """Every set of at most `max_losses` lost ranks, smallest first (a cover plan's domain)."""
    return [c for k in range(1, max_losses + 1) for c in itertools.combinations(range(world), k)]
