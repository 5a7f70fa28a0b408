"""A rank's view of its engine's membership: the epoch, the fault flag, and the staged change.

``stage_change`` runs when a ``Change`` reaches the rank (on the daemon connection's thread): the
fault flag goes up and the change waits for the step boundary. ``at_boundary`` applies it: the
epoch moves on and the fault clears. Every transition is recorded with a monotonic timestamp
(``trace``), which is how a change's pause is measured on the rank's side.

Reference parity: Runtime.on_change / at_boundary of core/everserve/comm/runtime.py:275-369 (the
collective swap itself lives in :mod:`everserve_b200.runtime.groups`).
"""

from __future__ import annotations

import threading
import time
from typing import Any


class Runtime:
    def __init__(self, rank: int, epoch: int = 0):
        self.rank = rank
        self.epoch = epoch
        self.fault = threading.Event()
        self.staged: Any = None
        self._lock = threading.Lock()
        self.events: list[tuple[float, str, dict]] = []

    def trace(self, what: str, **kv) -> None:
        with self._lock:
            self.events.append((time.monotonic(), what, kv))
            del self.events[:-1024]

    def stage_change(self, change) -> None:
        with self._lock:
            self.staged = change
        self.fault.set()
        self.trace("staged", epoch=getattr(change, "epoch", None))

    def at_boundary(self, epoch: int) -> None:
        with self._lock:
            self.epoch = epoch
            self.staged = None
        self.fault.clear()
        self.trace("boundary", epoch=epoch)

    @property
    def pending(self) -> bool:
        return self.fault.is_set()
