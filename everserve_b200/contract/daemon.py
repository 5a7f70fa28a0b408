"""The process side of the node daemon's Unix socket: workers, spares, heads and clients.

Every process of an engine holds one connection to its node's daemon (``everserve-node``) and
speaks ``signals.Signal`` frames (4-byte big-endian length + payload, :mod:`everserve_b200.wire`).

* :class:`DaemonConnection` - a worker or a spare. It registers (``Register`` with the role, rank,
  device, protocol range, host), then a reader thread serves what the daemon sends:

  - ``Change``: the participant's ``on_change`` runs (a spare restores the lost rank's KV there)
    and the connection answers ``Ack{rank, epoch, error}``; the daemon collects the acks and the
    coordinator commits or abandons the change;
  - ``MembershipCommitted``: recorded; a worker that the new membership no longer places on this
    node and device is displaced (``on_displaced``);
  - ``Notice``, ``Abandoned``, ``CoverPlan``, ``GroupId``, ``Join`` (to the participant),
    ``DumpStacks`` (answered with every thread's stack), engine policy / placement / state.

  Calls: ``report_lost`` (``RankLost`` up to the coordinator), ``notice``, ``join`` (an opaque
  offer to the head), ``report`` (cover group reports), ``report_leak``, ``goodbye``.
* :class:`DaemonClient` - the head (``ROLE_HEAD``) or a client (``ROLE_CLIENT``): hears every
  change of the engine (``Change``, ``MembershipCommitted``, ``Abandoned``) in order and can wait
  for the next commit; sends ``Join`` offers to ranks and ``ReplayOffer``s.
* :class:`UndecidedConnection` - a process that asks the coordinator for its role
  (``ROLE_UNDECIDED``) and waits for ``RoleAssigned``.

Reference parity: ``core/everserve/contract/daemon.py:78-1009`` (Participant, HearsEngine,
DaemonConnection, DaemonClient, UndecidedConnection, dump_stacks, ask_replay, GroupIds); the
signals are the same messages, so these connections speak to the reference's daemon and the
daemon here speaks to the reference's processes.
"""

from __future__ import annotations

import os
import queue
import socket
import sys
import threading
import time
import traceback
from dataclasses import dataclass, field
from typing import Any, Callable, Protocol, Sequence

from .. import wire
from ..proto import signals as sp

PROTOCOL = sp.PROTOCOL_VERSION
PROTOCOL_OLDEST = sp.PROTOCOL_OLDEST


class Refused(RuntimeError):  # noqa: N818 - the daemon's word
    """The daemon refused this process (protocol range, role, or a stale epoch)."""


class Participant(Protocol):
    """What a worker or spare offers its connection (all callbacks run on the reader thread)."""

    def identity(self) -> tuple[int, int]:
        """(rank, device)."""

    def on_change(self, change: Any) -> str | None:
        """A membership change names this process: stage it. Returns an error string or None."""

    def on_notice(self, rank: int, deadline_ms: int) -> None: ...

    def on_abandoned(self, epoch: int, detail: str) -> None: ...

    def on_committed(self, committed: Any) -> None: ...

    def on_join(self, join: Any) -> None: ...

    def on_displaced(self, epoch: int, why: str) -> None: ...


def own_host() -> str:
    return os.environ.get("EVERSERVE_HOST") or socket.gethostname()


def dump_stacks() -> str:
    """Every Python thread's stack, as text (the answer to ``DumpStacks``)."""
    out = []
    names = {t.ident: t.name for t in threading.enumerate()}
    for ident, frame in sys._current_frames().items():
        out.append(f"--- thread {names.get(ident, '?')} ({ident})\n")
        out.extend(traceback.format_stack(frame))
    return "".join(out)


def _kind(sig) -> str | None:
    return sig.WhichOneof("kind")


class _Link:
    """One framed connection to the daemon with a reader thread and a send lock."""

    def __init__(self, path: str, timeout_s: float = 10.0):
        self.path = path
        deadline = time.monotonic() + timeout_s
        while True:
            try:
                self.sock = wire.connect(path, timeout=timeout_s)
                break
            except OSError:
                if time.monotonic() > deadline:
                    raise
                time.sleep(0.05)
        self.sock.settimeout(None)
        self._send_lock = threading.Lock()
        self.closed = threading.Event()

    def send(self, sig) -> None:
        data = sig.SerializeToString()
        with self._send_lock:
            wire.send(self.sock, data)

    def recv(self):
        s = sp.Signal()
        s.ParseFromString(wire.recv(self.sock))
        return s

    def close(self) -> None:
        self.closed.set()
        try:
            self.sock.shutdown(socket.SHUT_RDWR)
        except OSError:
            pass
        self.sock.close()


class HearsEngine:
    """Engine-wide facts the daemon relays: policy, placement and instance state."""

    def __init__(self):
        self._facts_cond = threading.Condition()
        self._policy = None
        self._placement = None
        self._state = None

    def _heard_fact(self, sig, kind: str) -> bool:
        with self._facts_cond:
            if kind == "engine_policy":
                self._policy = sig.engine_policy
            elif kind == "engine_placement":
                self._placement = sig.engine_placement
            elif kind == "instance_state":
                self._state = sig.instance_state
            else:
                return False
            self._facts_cond.notify_all()
        return True

    def state(self):
        return self._state

    def placement(self):
        return self._placement

    def policy_signal(self):
        return self._policy

    def engine_placement(self, timeout_s: float | None = None):
        with self._facts_cond:
            if not self._facts_cond.wait_for(lambda: self._placement is not None, timeout=timeout_s):
                raise TimeoutError("no engine placement heard")
            return self._placement


class DaemonConnection(HearsEngine):
    """A worker's or spare's connection (see the module doc)."""

    def __init__(self, path: str, engine: str, participant: Participant, role: int = sp.ROLE_WORKER,
                 any_rank: bool = False, stage: Sequence[int] = (), timeout_s: float = 10.0, node: str = "",
                 identity=None, compile_cache=None):
        super().__init__()
        self.engine_name = engine
        self.participant = participant
        self.role = role
        self.epoch = 0
        self.committed = None
        self._link = _Link(path, timeout_s)
        rank, device = participant.identity()
        self.rank, self.device = rank, device
        self.node = node or os.environ.get("EVERSERVE_NODE", "")
        reg = sp.Register(engine=engine, rank=rank, role=role, any_rank=any_rank, protocol=PROTOCOL,
                          protocol_oldest=PROTOCOL_OLDEST, launcher_pid=os.getpid(), host=own_host(),
                          stage=list(stage), member=sp.Member(node=self.node, device=device))
        if identity is not None:
            reg.identity.CopyFrom(identity)
        if compile_cache is not None:  # the pair of the artifacts this process loads (compile_cache.py)
            reg.compile_cache.CopyFrom(compile_cache)
        self._link.send(sp.Signal(register=reg))
        self._reader = threading.Thread(target=self._serve, name=f"daemon-{engine}-{rank}", daemon=True)
        self._reader.start()

    # ---- calls -----------------------------------------------------------------------------------
    def report_lost(self, ranks: Sequence[int], detail: str = "", epoch: int = 0,
                    reason: int = sp.REASON_UNSPECIFIED) -> None:
        self._link.send(sp.Signal(rank_lost=sp.RankLost(ranks=list(ranks), detail=detail, epoch=epoch or self.epoch,
                                                        reason=reason)))

    def notice(self, rank: int, deadline_ms: int, reason: int = sp.REASON_NOTICE) -> None:
        self._link.send(sp.Signal(notice=sp.Notice(rank=rank, deadline_ms=deadline_ms, reason=reason)))

    def join(self, epoch: int, payload: bytes) -> None:
        """An opaque message to the engine's head (relayed by daemon -> coordinator -> daemon)."""
        self._link.send(sp.Signal(join=sp.Join(engine=self.engine_name, epoch=epoch, rank=self.rank, payload=payload)))

    def report(self, report) -> None:
        name = type(report).DESCRIPTOR.name
        key = {"GroupFormed": "group_formed", "GroupFailed": "group_failed", "GroupReleased": "group_released",
               "GroupReady": "group_ready"}[name]
        self._link.send(sp.Signal(**{key: report}))

    def report_group_id(self, gid) -> None:
        self._link.send(sp.Signal(group_id=gid))

    def report_leak(self, release: str, run_s: float, leaked_total: int) -> None:
        self._link.send(sp.Signal(release_leaked=sp.ReleaseLeaked(
            engine=self.engine_name, rank=self.rank, release=release, run_ms=int(run_s * 1000),
            leaked_total=leaked_total)))

    def goodbye(self, cause: int = sp.STOP_CAUSE_STOPPED, detail: str = "") -> None:
        try:
            self._link.send(sp.Signal(goodbye=sp.Goodbye(cause=cause, detail=detail)))
        except OSError:
            pass

    def close(self, cause: int = sp.STOP_CAUSE_STOPPED) -> None:
        self.goodbye(cause)
        self._link.close()

    # ---- the reader ------------------------------------------------------------------------------
    def _serve(self) -> None:
        while not self._link.closed.is_set():
            try:
                sig = self._link.recv()
            except (ConnectionError, OSError):
                return
            kind = _kind(sig)
            p = self.participant  # a spare for any rank hands its link to the rank it became
            try:
                if kind == "change":
                    ch = sig.change
                    err = p.on_change(ch)
                    if not err:
                        self.epoch = max(self.epoch, ch.epoch)
                    self._link.send(sp.Signal(ack=sp.Ack(rank=self.rank, epoch=ch.epoch, error=err or "")))
                elif kind == "membership_committed":
                    mc = sig.membership_committed
                    self.epoch = max(self.epoch, mc.epoch)
                    self.committed = mc
                    mine = [m for m in mc.members if m.rank == self.rank]
                    if self.role == sp.ROLE_WORKER and mine and mine[0].node and self.node and (
                            mine[0].node != self.node or (mine[0].HasField("device") and mine[0].device != self.device)):
                        p.on_displaced(mc.epoch, f"rank {self.rank} is held by {mine[0].node}:{mine[0].device}")
                    if self.role == sp.ROLE_SPARE and mine and mine[0].node == self.node and (
                            not mine[0].HasField("device") or mine[0].device == self.device):
                        self.role = sp.ROLE_WORKER
                    p.on_committed(mc)
                elif kind == "notice":
                    p.on_notice(sig.notice.rank, sig.notice.deadline_ms)
                elif kind == "abandoned":
                    p.on_abandoned(sig.abandoned.epoch, sig.abandoned.detail)
                elif kind == "join":
                    p.on_join(sig.join)
                elif kind == "dump_stacks":
                    self._link.send(sp.Signal(stacks_dumped=sp.StacksDumped(
                        request_id=sig.dump_stacks.request_id, text=dump_stacks())))
                elif kind == "goodbye":
                    p.on_abandoned(self.epoch, f"refused by the daemon: {sig.goodbye.detail}")
                elif kind == "cover_plan" and hasattr(p, "on_cover_plan"):
                    p.on_cover_plan(sig.cover_plan)
                elif kind == "group_id" and hasattr(p, "on_group_id"):
                    p.on_group_id(sig.group_id)
                else:
                    self._heard_fact(sig, kind or "")
            except (ConnectionError, OSError):
                return
            except Exception:  # noqa: BLE001 - a participant's failure must not end the link
                traceback.print_exc()


@dataclass
class Heard:
    """One change as a head hears it."""

    epoch: int
    kind: str  # "change" | "committed" | "abandoned"
    change: Any = None
    committed: Any = None
    detail: str = ""
    at: float = field(default_factory=time.monotonic)


class DaemonClient(HearsEngine):
    """The head's (or a client's) connection: hears the engine's changes and joins."""

    def __init__(self, path: str, engine: str, role: int = sp.ROLE_HEAD, timeout_s: float = 10.0, node: str = "",
                 on_heard: Callable[[Heard], None] | None = None):
        super().__init__()
        self.engine_name = engine
        self._link = _Link(path, timeout_s)
        self.node = node or os.environ.get("EVERSERVE_NODE", "")
        self._link.send(sp.Signal(register=sp.Register(
            engine=engine, role=role, protocol=PROTOCOL, protocol_oldest=PROTOCOL_OLDEST, launcher_pid=os.getpid(),
            host=own_host(), member=sp.Member(node=self.node))))
        self.heard: queue.Queue[Heard] = queue.Queue()
        self.joins: queue.Queue = queue.Queue()
        self.replay_asks: queue.Queue = queue.Queue()
        self.epoch = 0
        self.pending_change = threading.Event()
        self.last_change = None
        self._on_heard = on_heard
        self._reader = threading.Thread(target=self._serve, name=f"daemon-client-{engine}", daemon=True)
        self._reader.start()

    def _serve(self) -> None:
        while not self._link.closed.is_set():
            try:
                sig = self._link.recv()
            except (ConnectionError, OSError):
                return
            kind = _kind(sig)
            h = None
            if kind == "change":
                self.last_change = sig.change
                self.pending_change.set()
                h = Heard(sig.change.epoch, "change", change=sig.change)
            elif kind == "membership_committed":
                mc = sig.membership_committed
                self.epoch = max(self.epoch, mc.epoch)
                h = Heard(mc.epoch, "committed", committed=mc)
            elif kind == "abandoned":
                h = Heard(sig.abandoned.epoch, "abandoned", detail=sig.abandoned.detail)
            elif kind == "join":
                self.joins.put(sig.join)
            elif kind == "replay_ask":
                self.replay_asks.put(sig.replay_ask)
            elif kind == "dump_stacks":
                try:
                    self._link.send(sp.Signal(stacks_dumped=sp.StacksDumped(
                        request_id=sig.dump_stacks.request_id, text=dump_stacks())))
                except OSError:
                    return
            else:
                self._heard_fact(sig, kind or "")
            if h is not None:
                self.heard.put(h)
                if self._on_heard is not None:
                    self._on_heard(h)

    def wait_committed(self, timeout_s: float | None = None, after_epoch: int = 0) -> Heard:
        """The next commit (or abandonment) above `after_epoch`; changes heard meanwhile are skipped."""
        deadline = None if timeout_s is None else time.monotonic() + timeout_s
        while True:
            left = None if deadline is None else max(0.0, deadline - time.monotonic())
            try:
                h = self.heard.get(timeout=left)
            except queue.Empty:
                raise TimeoutError(f"no membership commit within {timeout_s} s") from None
            if h.kind in ("committed", "abandoned") and h.epoch > after_epoch:
                self.pending_change.clear()
                return h

    def join(self, rank: int, epoch: int, payload: bytes) -> None:
        self._link.send(sp.Signal(join=sp.Join(engine=self.engine_name, epoch=epoch, rank=rank, payload=payload)))

    def next_join(self, timeout_s: float | None = None):
        try:
            return self.joins.get(timeout=timeout_s)
        except queue.Empty:
            raise TimeoutError(f"no join within {timeout_s} s") from None

    def report_lost(self, ranks: Sequence[int], detail: str = "", epoch: int = 0) -> None:
        self._link.send(sp.Signal(rank_lost=sp.RankLost(ranks=list(ranks), detail=detail, epoch=epoch or self.epoch)))

    def notice(self, rank: int, deadline_ms: int) -> None:
        self._link.send(sp.Signal(notice=sp.Notice(rank=rank, deadline_ms=deadline_ms, reason=sp.REASON_NOTICE)))

    def offer_replay(self, ask, handle: str) -> None:
        """Answer a spare's ``ReplayAsk`` with a handle to the head's start-up record."""
        self._link.send(sp.Signal(replay_offer=sp.ReplayOffer(engine=ask.engine, rank=ask.rank, handle=handle,
                                                              to=ask.asker)))

    def goodbye(self, cause: int = sp.STOP_CAUSE_STOPPED, detail: str = "") -> None:
        try:
            self._link.send(sp.Signal(goodbye=sp.Goodbye(cause=cause, detail=detail)))
        except OSError:
            pass

    def close(self) -> None:
        self.goodbye()
        self._link.close()


class UndecidedConnection(HearsEngine):
    """A process that lets the coordinator choose its role (``ROLE_UNDECIDED``)."""

    def __init__(self, path: str, engine: str, rank: int = 0, device: int = 0, timeout_s: float = 10.0, node: str = ""):
        super().__init__()
        self._link = _Link(path, timeout_s)
        self.node = node or os.environ.get("EVERSERVE_NODE", "")
        self._link.send(sp.Signal(register=sp.Register(
            engine=engine, rank=rank, role=sp.ROLE_UNDECIDED, protocol=PROTOCOL, protocol_oldest=PROTOCOL_OLDEST,
            launcher_pid=os.getpid(), host=own_host(), member=sp.Member(node=self.node, device=device))))

    def assigned(self, timeout_s: float | None = None):
        """The coordinator's answer; raises :class:`Refused` for a refusal."""
        self._link.sock.settimeout(timeout_s)
        try:
            while True:
                sig = self._link.recv()
                if _kind(sig) == "role_assigned":
                    ra = sig.role_assigned
                    if ra.refusal:
                        raise Refused(ra.refusal)
                    return ra
                self._heard_fact(sig, _kind(sig) or "")
        except socket.timeout:
            raise TimeoutError(f"no role within {timeout_s} s") from None
        finally:
            self._link.sock.settimeout(None)

    def close(self) -> None:
        self._link.close()
