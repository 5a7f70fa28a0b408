"""Forms the communicator groups a coordinator's cover plan names, before any loss.

The coordinator plans, for every standing spare, the member set in which it holds the position it
stands for, and lists the groups each set needs (one pipeline group per tensor column when the
engine has stages; tensor-parallel groups are member tables over peer memory and need none). Every
process forms, in background threads, the planned groups it is a member of, under the rendezvous
prefix ``cover/g<generation>/<spans>/``, and reports each one formed (or failed) through its
daemon; the coordinator counts a set covered once every member of every group reported it. When
a change makes a planned set the engine's membership, the boundary adopts the pre-formed group
(``take``) instead of forming one while the engine waits. Groups a newer plan no longer names are
released and reported.

Members are named by a text key: a rank position (``"1"``) or a spare by the position it stands
for and where it runs (``"R1@n0:2"``).

Reference parity: Cover of core/everserve/comm/cover.py:183-650 (apply, background formation,
reports, release) over this framework's epoch groups.
"""

from __future__ import annotations

import datetime
import threading
import time
from typing import Callable

import torch
import torch.distributed as dist

from ..proto import signals as sp


def member_key(m) -> str:
    """Text key of a signals.SetMember."""
    if m.WhichOneof("kind") == "spare":
        return f"R{m.spare.for_rank}@{m.spare.node}:{m.spare.device}"
    return str(m.rank)


def _form_pg(store, prefix: str, rank: int, size: int, device: torch.device, timeout_s: float):
    ps = dist.PrefixStore(prefix, store)
    t = datetime.timedelta(seconds=timeout_s)
    if device.type == "cuda":
        opts = dist.ProcessGroupNCCL.Options()
        opts._timeout = t
        return dist.ProcessGroupNCCL(ps, rank, size, opts)
    return dist.ProcessGroupGloo(ps, rank, size, t)


class Cover:
    def __init__(self, store, me: str, engine: str, device: torch.device,
                 report: Callable[[object], None] | None = None, timeout_s: float = 30.0):
        """`store`: the rendezvous store, or a function making a client of it. A store client
        serves one blocking request at a time, so formations that run beside each other (and
        beside the boundary's own) each need a client of their own: one formation waiting for a
        peer's key must not hold up another's writes, or two processes wait on each other."""
        self.store, self.me, self.engine, self.device = store, me, engine, device
        self.report = report
        self.timeout_s = timeout_s
        self._lock = threading.Lock()
        self.held: dict[str, tuple[object, int, list]] = {}  # spans key -> (group, generation, spans)
        self.forming: set[str] = set()
        self.generation = 0
        self.events: list[tuple[float, str, str]] = []
        self._frozen = False
        self._latest = None

    def freeze(self) -> None:
        """A change is under way: hold every group (a plan arriving now is applied at unfreeze)."""
        with self._lock:
            self._frozen = True

    def unfreeze(self) -> None:
        with self._lock:
            self._frozen = False
            plan, self._latest = self._latest, None
        if plan is not None:
            self.apply(plan)

    def has(self, keys: list[str]) -> bool:
        with self._lock:
            return ",".join(keys) in self.held

    def set_me(self, me: str) -> None:
        """A spare that took a rank is that rank in later plans."""
        self.me = me

    def apply(self, plan) -> None:
        with self._lock:
            if self._frozen:
                self._latest = plan
                return
        self.generation = plan.generation
        wanted = {}
        for g in plan.groups:
            keys = [member_key(m) for m in g.spans]
            if self.me not in keys:
                continue
            wanted[",".join(keys)] = (g, keys)
        with self._lock:
            # a group of an older plan is formed again: the process behind a position may have
            # changed since (a spare took it), and a group with a dead member is no cover
            stale = [k for k, v in self.held.items() if k not in wanted or v[1] != plan.generation]
        for k in stale:
            self._release(k)
        with self._lock:
            todo = [(k, g, keys) for k, (g, keys) in wanted.items() if k not in self.held and k not in self.forming]
            for k, _, _ in todo:
                self.forming.add(k)
        for k, g, keys in todo:
            threading.Thread(target=self._form, args=(plan.generation, k, g, keys), name=f"cover-{k}",
                             daemon=True).start()

    def _form(self, generation: int, key: str, g, keys: list[str]) -> None:
        t0 = time.monotonic()
        rank = keys.index(self.me)
        try:
            store = self.store() if callable(self.store) else self.store
            pg = _form_pg(store, f"cover/g{generation}/{key}/", rank, len(keys), self.device, self.timeout_s)
            # a first collective, so the group is usable (not only created) when a change adopts it
            t = torch.zeros(1, device=self.device)
            pg.allreduce([t]).wait()
        except Exception as e:  # noqa: BLE001 - reported; the boundary then forms its own group
            with self._lock:
                self.forming.discard(key)
            self.events.append((time.monotonic(), "failed", key))
            self._send(sp.GroupFailed(engine=self.engine, generation=generation, spans=list(g.spans), scope=g.scope,
                                      error=str(e), member=self._me_member(g.spans)))
            return
        with self._lock:
            self.forming.discard(key)
            self.held[key] = (pg, generation, list(g.spans))
        self.events.append((time.monotonic(), "formed", key))
        self._send(sp.GroupFormed(engine=self.engine, generation=generation, spans=list(g.spans), scope=g.scope,
                                  seconds=time.monotonic() - t0, member=self._me_member(g.spans)))

    def _me_member(self, spans):
        for m in spans:
            if member_key(m) == self.me:
                return m
        return sp.SetMember()

    def _release(self, key: str) -> None:
        with self._lock:
            entry = self.held.pop(key, None)
        if entry is None:
            return
        pg, generation, spans = entry
        if hasattr(pg, "abort"):
            try:
                pg.abort()
            except Exception:  # noqa: BLE001
                pass
        self.events.append((time.monotonic(), "released", key))
        self._send(sp.GroupReleased(engine=self.engine, generation=generation, spans=spans,
                                    scope=sp.SCOPE_FABRIC, member=self._me_member(spans)))

    def _send(self, report) -> None:
        if self.report is not None:
            try:
                self.report(report)
            except OSError:
                pass

    def take(self, keys: list[str]):
        """The pre-formed group over exactly these members (in this order), handed over; or None."""
        with self._lock:
            entry = self.held.pop(",".join(keys), None)
        if entry is None:
            return None
        self.events.append((time.monotonic(), "taken", ",".join(keys)))
        return entry[0]

    def close(self) -> None:
        for k in list(self.held):
            self._release(k)
