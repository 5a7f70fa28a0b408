"""The committed-KV protocol: what a rank's KV persistence must offer the runtime.

A step's K/V rows are saved per layer as the forward writes them, committed once the step ends
(the step number, the membership epoch, and each request's committed token count), and fenced: a
rank waits until step s - depth has been acknowledged before it may run further ahead. A spare
taking a lost rank restores that rank's rows and counts, optionally only rows written since a
step it already holds.

Reference parity: the CommittedKV protocol of core/everserve/state/committed.py:33-109.
"""

from __future__ import annotations

from typing import Mapping, Protocol, Sequence

import torch


class CommittedKV(Protocol):
    def save(self, layer: int, kv: torch.Tensor, slots: torch.Tensor) -> None:
        """Note that `layer`'s cache holds new rows at `slots` this step."""

    def commit(self, epoch: int, step: int, counts: Mapping[str, int], slots: torch.Tensor | None = None) -> None:
        """The step is complete: persist its rows and the requests' committed token counts."""

    def fence(self, step: int, timeout_s: float = 30.0) -> None:
        """Block until `step` is acknowledged by the store (a no-op for steps below the first)."""

    def committed(self, request_id: str) -> int:
        """Tokens of `request_id` whose K/V is committed."""

    def stats(self) -> Mapping[str, float]: ...

    def timeline(self) -> Sequence[Mapping[str, float]]: ...

    def evicted(self, request_id: str, kept_tokens: int) -> None: ...

    def finished(self, request_id: str) -> None: ...

    def clear(self) -> None: ...

    def restore(self, dead_rank: int, moves: Mapping[int, int] | None = None, since_step: int = 0) -> dict[str, int]:
        """Write `dead_rank`'s committed rows into this rank's cache; returns the committed counts."""
