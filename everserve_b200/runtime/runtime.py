"""A rank's view of its engine's membership: the epoch, the fault flag, and the staged change.

``stage_change`` runs when a ``Change`` reaches the rank (on the daemon connection's thread): the
fault flag goes up and the change waits for the step boundary. ``at_boundary`` applies it: the
epoch moves on and the fault clears. Every transition is recorded with a monotonic timestamp
(``trace``), which is how a change's pause is measured on the rank's side.

With ``EVERSERVE_EVENT_DIR`` set, every transition is also appended as one JSON line (thread,
monotonic and wall time) to ``rank<N>.trace.jsonl`` there, and ``dump()`` writes the last 4096 as
``rank<N>.json``, written beside and renamed over so a reader never sees a torn file.

Reference parity: Runtime.on_change / at_boundary of core/everserve/comm/runtime.py:275-369 and its
event log (runtime.py:141-169, 612-632); the collective swap itself lives in
:mod:`everserve_b200.runtime.groups`.
"""

from __future__ import annotations

import json
import os
import threading
import time
from typing import Any


class Runtime:
    KEEP = 4096

    def __init__(self, rank: int, epoch: int = 0, event_dir: str | None = None):
        self.rank = rank
        self.epoch = epoch
        self.fault = threading.Event()
        self.staged: Any = None
        self._lock = threading.Lock()
        self.events: list[tuple[float, str, dict]] = []
        self.event_dir = event_dir if event_dir is not None else os.environ.get("EVERSERVE_EVENT_DIR", "")
        self._trace_file = None
        if self.event_dir:
            os.makedirs(self.event_dir, exist_ok=True)
            self._trace_file = open(os.path.join(self.event_dir, f"rank{rank}.trace.jsonl"), "a", buffering=1)  # noqa: SIM115

    def trace(self, what: str, **kv) -> None:
        t = time.monotonic()
        with self._lock:
            self.events.append((t, what, kv))
            del self.events[: -self.KEEP]
            if self._trace_file is not None:
                rec = {"at": t, "wall": time.time(), "thread": threading.current_thread().name, "kind": what,
                       "epoch": self.epoch, **kv}
                self._trace_file.write(json.dumps(rec, default=str) + "\n")

    def dump(self) -> str | None:
        """Write the kept events as ``rank<N>.json`` in the event directory; returns its path."""
        if not self.event_dir:
            return None
        with self._lock:
            rows = [{"at": t, "kind": w, **kv} for t, w, kv in self.events]
        final = os.path.join(self.event_dir, f"rank{self.rank}.json")
        tmp = final + ".part"
        with open(tmp, "w") as f:
            json.dump(rows, f, default=str)
        os.replace(tmp, final)
        return final

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
