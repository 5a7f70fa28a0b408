"""Helpers for an engine's head: who launched it, why it stopped, and waiting for a commit.

Reference parity: core/everserve/contract/head.py:34-86.
"""

from __future__ import annotations

import os

from ..proto import signals as sp


class ChangeAbandoned(RuntimeError):
    """The coordinator abandoned the change: the engine is down."""

    def __init__(self, epoch: int, detail: str):
        super().__init__(f"membership change to epoch {epoch} abandoned: {detail}")
        self.epoch, self.detail = epoch, detail


def launcher_pid(env_var: str = "EVERSERVE_LAUNCHER_PID") -> int:
    """The pid the daemon should watch for this engine: the launcher's when one set it, else ours."""
    v = os.environ.get(env_var, "")
    return int(v) if v.isdigit() else os.getpid()


def stop_cause(failure: str | None) -> tuple[int, str]:
    """The Goodbye for a head that stops: STOPPED on a clean exit, FAILED with the failure text."""
    if not failure:
        return sp.STOP_CAUSE_STOPPED, ""
    return sp.STOP_CAUSE_FAILED, failure[:1024]


def wait_commit(client, timeout_s: float | None = None, after_epoch: int = 0):
    """The next MembershipCommitted a DaemonClient hears; raises ChangeAbandoned on Abandoned."""
    h = client.wait_committed(timeout_s=timeout_s, after_epoch=after_epoch)
    if h.kind == "abandoned":
        raise ChangeAbandoned(h.epoch, h.detail)
    return h.committed
