"""Placement plans: which rank owns which unit of work, before and after a loss.

A unit is a piece of the model that can move between ranks without changing any tensor shape: a
KV head with its query heads, a fixed-width slice of the MLP's intermediate dimension, a
fixed-size chunk of experts. A plan is a pure function of the world and the lost ranks, so every
survivor computes the same plan without being told.

Reference parity: core/everserve/reference/plan.py:27-129 (the same functions and rules).
"""

from __future__ import annotations

from typing import Callable, Hashable, Sequence

Owned = dict


def even_units(n_units: int, world: int) -> dict[int, list[int]]:
    """Unit indices split evenly across ranks, in rank order (an uneven split is refused)."""
    if world <= 0:
        raise ValueError(f"world must be positive, got {world}")
    if n_units % world:
        raise ValueError(f"{n_units} units do not divide evenly over {world} ranks")
    k = n_units // world
    return {r: list(range(r * k, (r + 1) * k)) for r in range(world)}


def expert_chunks(n_experts: int, world: int, chunk: int) -> dict[int, list[tuple[int, ...]]]:
    """Experts grouped into fixed-size chunks, each rank its contiguous share of chunks."""
    if chunk <= 0:
        raise ValueError(f"chunk must be positive, got {chunk}")
    if world <= 0 or n_experts % world:
        raise ValueError(f"{n_experts} experts do not divide evenly over {world} ranks")
    per = n_experts // world
    if per % chunk:
        raise ValueError(f"{per} experts per rank do not divide into chunks of {chunk}")
    return {r: [tuple(range(r * per + i, r * per + i + chunk)) for i in range(0, per, chunk)] for r in range(world)}


def after_loss(owned: dict[int, list[Hashable]], lost: Sequence[int],
               cost: Callable[[int, dict], object] | None = None) -> dict[int, list[Hashable]]:
    """The survivors' plan: every lost rank's units, in order, go one by one to the survivor with
    the least load (its unit count, or `cost`), the lowest rank on a tie."""
    lost = set(lost)
    new = {r: list(u) for r, u in owned.items() if r not in lost}
    if not new:
        raise ValueError("no survivor to take the units")
    cost = cost or (lambda r, o: len(o[r]))
    for dead in sorted(lost):
        for unit in owned.get(dead, []):
            r = min(new, key=lambda q: (cost(q, new), q))
            new[r].append(unit)
    return new


def moved(before: dict[int, list], after: dict[int, list]) -> dict[int, list]:
    """Units each survivor gained."""
    return {r: [u for u in after[r] if u not in set(before.get(r, []))] for r in after}


def capacity_after_one_loss(n_units: int, world: int, per_rank_capacity: int) -> bool:
    """Whether any single loss leaves the survivors room for every unit."""
    if world <= 1:
        return False
    need = -(-n_units // (world - 1))
    return need <= per_rank_capacity
