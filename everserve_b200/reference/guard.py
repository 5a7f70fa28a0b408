"""The reference tier's step guard: every survivor accepts a step, or every survivor re-runs it.

The product path applies a change between steps (``Runtime.at_boundary``) and replays what the
change cost from committed counts. The reference tier instead checks a stronger property on CPU
ranks: a rank may die in the middle of a step, after some of its collectives, and the survivors
still produce the same outputs bit for bit. ``StepGuard.run_step`` runs a step as an attempt:

* every collective of the step goes through ``all_reduce``, which refuses once a fault is
  flagged, stops waiting when one is flagged during the collective, and keeps the attempt's
  buffers;
* the commit callbacks record what the step wrote (the committed store keeps rows by step, so a
  re-run replaces and never duplicates);
* the attempt ends with the agreement all-reduce of a one per member: a sum of ``n`` accepts it;
* an attempt that fails (a collective error with a dead peer, a refused collective, a short
  agreement) is abandoned: its buffers are quarantined for two epochs (a group that cannot abort
  may still write into them), the abandon callbacks roll back what it wrote, and, once the fault
  is confirmed on the fault channel (bounded), the survivors recover and the step runs again;
* a recovery: ``leave`` moves the group to the survivors; the survivors exchange their accepted
  counts; a member that accepted a step the others did not (the agreement completed for some
  members only) rewinds to before it; ``absorb`` takes the lost ranks' units with their KV up to
  the last step every survivor accepted; the member that rewound then replays that step (output
  discarded) under the new placement, so the others' re-run of it has its partners.

Reference parity: Runtime.run_step / _agree / _reconcile_accepted / _abandon_attempt / quarantine
of core/everserve/comm/runtime.py:455-601 (the reference guard the CPU spec runs under).
"""

from __future__ import annotations

import threading
import time
from typing import Any, Callable, TypeVar

import torch

T = TypeVar("T")


class StepAborted(RuntimeError):
    """A collective was refused because a fault is flagged."""


class StepGuard:
    def __init__(self, group, leave: Callable[[dict], None], absorb: Callable[[dict, int], None], faults=None,
                 confirm_timeout_s: float = 10.0):
        """`group`: the members' group (``all_reduce``, ``size``, ``rank``; moved by `leave`).
        `leave(fault)`: moves the group to the survivors. `absorb(fault, upto_step)`: takes the
        lost ranks' units, their KV up to step `upto_step` (-1: none).
        `faults`: a queue-like source of fault messages (``next(timeout)``), read on a thread."""
        self.group = group
        self.leave = leave
        self.absorb = absorb
        self.confirm_timeout_s = confirm_timeout_s
        self.epoch = 0
        self.accepted = 0
        self.fault: dict | None = None
        self.lock = threading.Lock()
        # attempt: an attempt starts; commit: its writes go to the committed store (before the
        # agreement, so a member that dies after it leaves them); abandon: roll the attempt's
        # writes back; accept: the step is accepted; replay: rewind to before the last accepted
        # step, which is about to run again (a member that is ahead replays it)
        self.attempt_callbacks: list[Callable[[], None]] = []
        self.commit_callbacks: list[Callable[[], None]] = []
        self.abandon_callbacks: list[Callable[[], None]] = []
        self.accept_callbacks: list[Callable[[], None]] = []
        self.replay_callbacks: list[Callable[[], None]] = []
        self.events: list[tuple[float, str, dict]] = []
        self._attempt_buffers: list[tuple[int, torch.Tensor]] = []
        self.quarantine: dict[int, list[torch.Tensor]] = {}
        self._last_fn: Callable[[], Any] | None = None
        if faults is not None:
            threading.Thread(target=self._watch, args=(faults,), name="fault-watch", daemon=True).start()

    def trace(self, what: str, **kv) -> None:
        self.events.append((time.monotonic(), what, kv))

    # ---- the fault channel ---------------------------------------------------------------------
    def _watch(self, faults) -> None:
        while True:
            try:
                f = faults.next(timeout=None)
            except Exception:  # noqa: BLE001 - the channel closed
                return
            self.flag(f)

    def flag(self, fault: dict) -> None:
        with self.lock:
            if fault.get("epoch", 0) > self.epoch:
                self.fault = fault

    # ---- collectives ---------------------------------------------------------------------------
    def all_reduce(self, t: torch.Tensor) -> torch.Tensor:
        with self.lock:
            if self.fault is not None:
                raise StepAborted("a fault is flagged")
            epoch = self.epoch
        self._attempt_buffers.append((epoch, t))
        start = getattr(self.group, "all_reduce_async", None)
        if start is None:
            return self.group.all_reduce(t)
        # a member whose ring neighbour left the collective (its own neighbour died) would wait
        # out the group's timeout; a fault flagged meanwhile ends the wait instead, and the buffer
        # stays in quarantine in case the old group writes into it later
        work = start(t)
        delay = 1e-4
        while not work.is_completed():
            if self.fault is not None:
                raise StepAborted("a fault was flagged while a collective waited")
            time.sleep(delay)
            delay = min(2 * delay, 2e-3)
        work.wait()
        return t

    def _agree(self, n: int) -> bool:
        t = torch.ones(1)
        self.all_reduce(t)
        return int(t.item()) == n

    # ---- attempts ------------------------------------------------------------------------------
    def _abandon(self) -> None:
        for epoch, t in self._attempt_buffers:
            self.quarantine.setdefault(epoch, []).append(t)
        self._attempt_buffers = []
        for old in [e for e in self.quarantine if e < self.epoch - 1]:
            del self.quarantine[old]
        for cb in self.abandon_callbacks:
            cb()

    def _wait_fault(self, timeout_s: float) -> bool:
        end = time.monotonic() + timeout_s
        while time.monotonic() < end:
            if self.fault is not None:
                return True
            time.sleep(0.005)
        return self.fault is not None

    def _recover(self) -> None:
        with self.lock:
            f, self.fault = self.fault, None
            self.epoch = max(self.epoch, int(f.get("epoch", self.epoch + 1)))
        self.trace("recover", lost=f.get("lost"), epoch=self.epoch, accepted=self.accepted)
        self.leave(f)
        n, me = self.group.size, self.group.rank
        counts = torch.zeros(n)
        counts[me] = float(self.accepted)
        self.group.all_reduce(counts)
        low = int(counts.min().item())
        self.trace("reconcile", accepted=self.accepted, low=low, counts=counts.tolist())
        if self.accepted > low + 1:
            raise RuntimeError(f"accepted {self.accepted} steps, another survivor only {low}")
        ahead = self.accepted > low
        if ahead:
            if self._last_fn is None:
                raise RuntimeError("a member is behind but there is no step to replay")
            for cb in self.replay_callbacks:  # back to before the step the others did not accept
                cb()
        self.absorb(f, low - 1)
        if ahead:
            self._last_fn()
            for cb in self.commit_callbacks:
                cb()
            if not self._agree(n):
                raise RuntimeError("the replayed step was not accepted by every member")
            self._attempt_buffers = []
            self.trace("replayed", accepted=self.accepted)

    def run_step(self, fn: Callable[[], T]) -> T:
        """Run `fn` (one step; its collectives through ``all_reduce``) until every survivor
        accepts it."""
        attempts = 0
        while True:
            if self.fault is not None:
                self._recover()
            for cb in self.attempt_callbacks:
                cb()
            n = self.group.size
            try:
                out = fn()
                for cb in self.commit_callbacks:
                    cb()
                ok = self._agree(n)
            except StepAborted:
                self.trace("aborted", attempt=attempts)
                self._abandon()
                attempts += 1
                continue
            except Exception as e:  # noqa: BLE001 - a fault only if the channel confirms one
                self.trace("failed", attempt=attempts, error=f"{type(e).__name__}: {e}"[:200])
                self._abandon()
                if self._wait_fault(self.confirm_timeout_s):
                    attempts += 1
                    continue
                raise
            if not ok:
                self._abandon()
                if not self._wait_fault(self.confirm_timeout_s):
                    raise RuntimeError("the step was not accepted and no fault came")
                attempts += 1
                continue
            self._attempt_buffers = []
            self.accepted += 1
            self._last_fn = fn
            for cb in self.accept_callbacks:
                cb()
            self.trace("accepted", accepted=self.accepted, attempts=attempts)
            return out
