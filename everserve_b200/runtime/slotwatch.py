"""The failure detector beside a rank: turns the collective kernels' late mask into lost ranks.

The peer-memory collective kernels bound every wait: a member that has not written its words
after ``bound_ns`` is named in the waiting rank's ``late`` word of the slot region (a bit per row)
and the kernel returns with a timeout status instead of hanging. ``SlotWatch`` is a thread that
polls that word (every 2 ms by default) and classifies each late member by its process:

* **dead** - ``/proc/<pid>`` is gone, a zombie, exiting (``PF_EXITING``), or has SIGKILL pending:
  the member is marked lost in the region at once and reported (``on_lost``, normally
  ``DaemonConnection.report_lost``);
* **hung** - alive but still late after ``hang_s``: reported the same way with the reason;
* a step-stall rule covers a member that died while this rank was not waiting on it: when the
  rank's step word shows a step in flight for longer than ``stall_s``, every member's process is
  checked.

Reference parity: SlotWatch of core/everserve/comm/slotwatch.py:52-281 (the same dead/hung rules
and the 2 ms poll) over this framework's slot region.
"""

from __future__ import annotations

import os
import threading
import time
from typing import Callable, Sequence

from ..parallel.slot import SlotRegion

_PF_EXITING = 0x4
_SIGKILL_BIT = 1 << (9 - 1)


def process_state(pid: int) -> str:
    """"dead", "exiting" or "alive" for a pid on this node (no such process reads as dead)."""
    if pid <= 0:
        return "dead"
    try:
        with open(f"/proc/{pid}/stat", "rb") as f:
            stat = f.read().decode(errors="replace")
    except (FileNotFoundError, ProcessLookupError):
        return "dead"
    except OSError:
        return "alive"
    rest = stat[stat.rfind(")") + 2 :].split()
    state = rest[0] if rest else "?"
    if state in ("Z", "X", "x"):
        return "dead"
    try:
        flags = int(rest[6])
    except (IndexError, ValueError):
        flags = 0
    if flags & _PF_EXITING:
        return "exiting"
    try:
        with open(f"/proc/{pid}/status") as f:
            for line in f:
                if line.startswith(("ShdPnd:", "SigPnd:")) and int(line.split()[1], 16) & _SIGKILL_BIT:
                    return "exiting"
    except OSError:
        return "dead"
    return "alive"


class SlotWatch:
    """Polls this rank's late word; reports dead members at once and hung ones after ``hang_s``."""

    def __init__(self, region: SlotRegion, row: int, on_lost: Callable[[list[int], str], None],
                 rank_of_row: Callable[[int], int] | None = None, members: Sequence[int] | None = None,
                 poll_s: float = 0.002, hang_s: float = 10.0, stall_s: float = 5.0, beat_limit_s: float = 0.0):
        self.region, self.row = region, row
        self.on_lost = on_lost
        self.rank_of_row = rank_of_row or (lambda r: r)
        self.members = list(members) if members is not None else None
        self.poll_s, self.hang_s, self.stall_s = poll_s, hang_s, stall_s
        self.beat_limit_s = beat_limit_s  # 0: heartbeats not watched
        self._beats: dict[int, tuple[int, float]] = {}  # row -> (last beat, when it changed)
        self.reported: set[int] = set()
        self.events: list[tuple[float, str, int]] = []
        self._late_since: dict[int, float] = {}
        self._step_since: tuple[int, float] | None = None
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._run, name=f"slotwatch-{row}", daemon=True)

    def start(self) -> "SlotWatch":
        self._thread.start()
        return self

    def stop(self) -> None:
        self._stop.set()
        if self._thread.is_alive():
            self._thread.join(timeout=1)

    def set_members(self, rows: Sequence[int]) -> None:
        self.members = list(rows)
        self.reported &= set(rows)
        self._late_since.clear()
        self._beats.clear()

    def _lost(self, rows: list[int], why: str) -> None:
        rows = [r for r in rows if r not in self.reported]
        if not rows:
            return
        now = time.monotonic()
        for r in rows:
            self.region.mark_lost(r)
            self.reported.add(r)
            self.events.append((now, why, r))
        self.on_lost([self.rank_of_row(r) for r in rows], why)

    def check(self) -> None:
        """One poll (the thread calls this every ``poll_s``)."""
        now = time.monotonic()
        late = self.region.late(self.row)
        rows = [r for r in range(8) if late >> r & 1 and r != self.row]
        if self.members is not None:
            rows = [r for r in rows if r in self.members]
        dead = []
        for r in rows:
            st = process_state(self.region.pid(r))
            if st != "alive":
                dead.append(r)
                continue
            t0 = self._late_since.setdefault(r, now)
            if now - t0 > self.hang_s:
                self._lost([r], "hung")
        for r in list(self._late_since):
            if r not in rows:
                del self._late_since[r]
        # a member whose heartbeat stopped is dead, late or not (its native beat thread ends only
        # with its process)
        if self.beat_limit_s > 0 and self.members is not None:
            for r in self.members:
                if r == self.row or r in dead or r in self.reported or self.region.pid(r) <= 0:
                    continue
                b = self.region.beat(r)
                last = self._beats.get(r)
                if last is None or last[0] != b:
                    self._beats[r] = (b, now)
                elif now - last[1] > self.beat_limit_s:
                    dead.append(r)
        if dead:
            self._lost(dead, "dead")
        # a step in flight too long: look at every member's process
        step = self.region.step(self.row)
        if step == 0:
            self._step_since = None
        elif self._step_since is None or self._step_since[0] != step:
            self._step_since = (step, now)
        elif now - self._step_since[1] > self.stall_s:
            members = self.members if self.members is not None else [r for r in range(8) if self.region.pid(r) > 0]
            gone = [r for r in members if r != self.row and process_state(self.region.pid(r)) != "alive"]
            if gone:
                self._lost(gone, "dead (step stalled)")

    def _run(self) -> None:
        while not self._stop.is_set():
            try:
                self.check()
            except Exception:  # noqa: BLE001 - the watcher must outlive a bad read
                pass
            time.sleep(self.poll_s)


def own_pid() -> int:
    return os.getpid()
