"""A shared/exclusive guard per communicator, so a release never frees a group under a call.

Calls on a group hold it shared; releasing (aborting, destroying) the group takes it exclusive and
waits, bounded, for the calls in flight. A release that times out leaves the group behind (it is
reported as leaked) instead of blocking the boundary.

Reference parity: core/everserve/comm/guard.py:24-69.
"""

from __future__ import annotations

import contextlib
import threading
import time


class Guard:
    def __init__(self):
        self._cond = threading.Condition()
        self._shared = 0
        self._exclusive = False

    @contextlib.contextmanager
    def shared(self):
        with self._cond:
            while self._exclusive:
                self._cond.wait()
            self._shared += 1
        try:
            yield
        finally:
            with self._cond:
                self._shared -= 1
                self._cond.notify_all()

    def exclusive(self, timeout_s: float | None = None) -> bool:
        """Take the guard exclusive (no new calls start); False if calls did not drain in time."""
        deadline = None if timeout_s is None else time.monotonic() + timeout_s
        with self._cond:
            self._exclusive = True
            while self._shared:
                left = None if deadline is None else deadline - time.monotonic()
                if left is not None and left <= 0:
                    return False
                self._cond.wait(left)
            return True

    def release_exclusive(self) -> None:
        with self._cond:
            self._exclusive = False
            self._cond.notify_all()

    @property
    def in_flight(self) -> int:
        return self._shared
