"""The head's executor for a multi-process engine, and its failover at a step boundary.

``MultiprocExecutor`` spawns one rank process per position (``everserve_b200.serving.rank``) plus
the spares, hosts the engine's rendezvous store (groups of every epoch form under ``e<epoch>/``)
and a carrier socket per rank, and registers with the node daemon as the engine's head
(``ROLE_HEAD``). Each step it sends the plan to every rank and collects the replies; the last
stage's column 0 returns the sampled ids.

When a rank is lost (its link ends, or a rank reports a failed step), the step raises
:class:`RankLost`. The failover step wrapper (:func:`failover`, installed with
``Engine.wrap_step``) then runs :meth:`MultiprocExecutor.complete_change`:

1. wait for the coordinator's ``MembershipCommitted`` (or ``Abandoned``: the engine is down);
   the coordinator has already delivered the ``Change`` to the survivors and to the spare, and the
   spare restored the lost rank's committed KV before it acked;
2. release departing ranks (a planned departure finishes its step and drains its commits);
3. offer a ``Join`` to each spare that took a rank (through the daemons and the coordinator) and
   wait for it to link;
4. ``boundary``: every member forms the new epoch's groups and reports what its cache holds;
5. resume: each running request's committed count is the minimum over the ranks, and the
   scheduler restarts every request at ``min(committed, n - 1)``; the uncommitted tail is replayed
   one position per step in decode shape, so the outputs are the no-fault outputs.

Reference parity: EverserveExecutor and its change completion of
adapters/vllm/everserve_vllm/executor.py:126-853 (cut step, new ring, boundary, join offers,
install, resume) and the step-loop hook of serving.py:44-86.
"""

from __future__ import annotations

import os
import secrets
import signal
import subprocess
import sys
import time
from dataclasses import dataclass, field

import torch.distributed as dist

from ..contract import join as joinfmt
from ..contract.daemon import DaemonClient
from ..engine.config import EngineConfig
from ..runtime.layout import ParallelLayout
from .carrier import CarrierServer, Link, LinkClosed, StepAbandoned


class RankLost(RuntimeError):
    def __init__(self, ranks, detail: str = ""):
        super().__init__(f"ranks {sorted(ranks)} lost: {detail}")
        self.ranks = sorted(ranks)
        self.detail = detail


class EngineDown(RuntimeError):
    """The coordinator abandoned the change: the engine cannot continue."""


@dataclass
class ChangeRecord:
    epoch: int
    lost: list
    outcome: int
    t_detect: float
    t_committed: float = 0.0
    t_joined: float = 0.0
    t_ready: float = 0.0
    t_resumed: float = 0.0
    t_fault: float = 0.0  # when the fault was injected (host-side injection only)
    t_fault_wall: float = 0.0  # the same instant on the wall clock (the coordinator's stamps are wall time)
    coordinator: dict = field(default_factory=dict)

    first_steps_ms: list = field(default_factory=list)  # device time of the steps after the resume

    def spans(self) -> dict:
        """The coordinator's part of the change, claim to commit, in ms: `decide` (loss reported to
        change delivered: outcome chosen, logged), `acks` (delivered to every node answering),
        `commit` (acknowledged to committed), and `claim_to_commit` in total.

        Reference parity: spans.claim_to_commit of adapters/vllm/everserve_vllm/spans.py:18."""
        c = self.coordinator
        rep, dlv, ack, com = (c.get(k) or 0 for k in ("reported_at_us", "delivered_at_us", "acknowledged_at_us",
                                                       "committed_at_us"))
        d = lambda a, b: round((b - a) / 1e3, 3) if a and b else None  # noqa: E731
        return {"decide": d(rep, dlv), "acks": d(dlv, ack), "commit": d(ack, com), "claim_to_commit": d(rep, com)}

    def as_dict(self) -> dict:
        """Milestones in ms from the fault when it is known (else from the head's detection)."""
        t0 = self.t_fault or self.t_detect
        ms = lambda t: round((t - t0) * 1e3, 3) if t else None  # noqa: E731
        return {"epoch": self.epoch, "lost": self.lost, "outcome": self.outcome, "from": "fault" if self.t_fault
                else "detect", "detected_ms": ms(self.t_detect), "committed_ms": ms(self.t_committed),
                "joined_ms": ms(self.t_joined), "ready_ms": ms(self.t_ready), "resumed_ms": ms(self.t_resumed),
                "coordinator": self.coordinator, "spans": self.spans(), "first_steps_ms": self.first_steps_ms}


class MultiprocExecutor:
    def __init__(self, cfg: EngineConfig, engine: str = "engine", daemon: str = "", store: str = "",
                 spares: tuple[int, ...] = (), device: str = "cpu", dtype: str = "float32", node: str = "",
                 env: dict | None = None, threads: int = 0, step_timeout_s: float = 300.0,
                 change_timeout_s: float = 120.0, log_dir: str | None = None, start_timeout_s: float = 600.0,
                 devices: list[int] | None = None, spare_places: list[dict] | None = None,
                 resident_spares: bool = False, local_ranks: list[int] | None = None):
        """`spare_places[i]`: where spare i runs when not on the head's node: its node's daemon
        and store sockets and the node name ({"daemon": ..., "store": ..., "node": ...}).
        `local_ranks`: the ranks this head starts itself (default: all); node agents
        (``everserve_b200.serving.node``) start the others on their nodes."""
        self.cfg = cfg
        self.engine = engine
        self._closed = False
        self.layout = ParallelLayout(cfg.tensor_parallel, cfg.pipeline_parallel)
        self.step_timeout_s = step_timeout_s
        self.change_timeout_s = change_timeout_s
        self.token = secrets.token_hex(16)
        self.carrier = CarrierServer(token=self.token)
        self.rdzv = dist.TCPStore("127.0.0.1", 0, is_master=True, wait_for_workers=False)
        self.rdzv_addr = f"127.0.0.1:{self.rdzv.port}"
        self.log_dir = log_dir
        self.procs: dict[str, subprocess.Popen] = {}
        self._logs = []
        base = [sys.executable, "-m", "everserve_b200.serving.rank", "--engine", engine, "--model", cfg.model.name,
                "--tp", str(cfg.tensor_parallel), "--pp", str(cfg.pipeline_parallel), "--device", device,
                "--dtype", dtype, "--seed", str(cfg.seed), "--block-size", str(cfg.block_size),
                "--max-batch", str(cfg.max_batch), "--max-model-len", str(cfg.max_model_len),
                "--rdzv", self.rdzv_addr, "--head", self.carrier.address]
        if cfg.num_blocks:
            base += ["--num-blocks", str(cfg.num_blocks)]
        if cfg.checkpoint:
            base += ["--checkpoint", cfg.checkpoint]
        self._startup_args = list(base[3:])  # the engine's configuration, for spares a daemon launches
        if daemon:
            base += ["--daemon", daemon]
        if store:
            base += ["--store", store]
        if node:
            base += ["--node", node]
        if threads:
            base += ["--threads", str(threads)]
        self.region = None
        self.rows = {r: r for r in range(self.layout.world)}  # rank position -> slot-region row
        gpu = self.gpu = device.startswith("cuda")
        if gpu and cfg.tensor_parallel > 1:
            from ..parallel.slot import MAX_ROWS, SlotRegion

            if self.layout.world + len(spares) > MAX_ROWS:
                raise ValueError(f"{self.layout.world} ranks + {len(spares)} spares exceed the region's {MAX_ROWS} rows")
            self.region_name = f"es_{engine}_{os.getpid()}_{secrets.token_hex(4)}"
            self.region = SlotRegion.create(self.region_name)
            base += ["--region", self.region_name]
            self._startup_args += ["--region", self.region_name]
        e = dict(os.environ)
        root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
        e["PYTHONPATH"] = os.pathsep.join([root] + [p for p in e.get("PYTHONPATH", "").split(os.pathsep) if p])
        # a rank's kernels load with its context, not at their first launch, so no step (a spare's
        # first one included) pays a module load that holds its member back at a collective
        e.setdefault("CUDA_MODULE_LOADING", "EAGER")
        e.update(env or {})
        e["EVERSERVE_CARRIER_TOKEN"] = self.token
        def dev_args(i: int) -> list[str]:
            if not gpu:
                return []
            return ["--device", f"cuda:{(devices or list(range(64)))[i]}"]

        # the head's daemon link first: ranks that node agents start elsewhere ask it for the
        # engine's start-up record before they can link
        self.client = DaemonClient(daemon, engine, node=node) if daemon else None
        self._next_row = self.layout.world + len(spares)
        if self.client is not None:
            import threading

            threading.Thread(target=self._answer_replays, name="replay-offers", daemon=True).start()
        self.local_ranks = list(range(self.layout.world)) if local_ranks is None else list(local_ranks)
        for r in self.local_ranks:
            self._spawn(f"rank{r}", base + ["--role", "worker", "--rank", str(r), "--row", str(r)] + dev_args(r), e)
        for i, r in enumerate(spares):
            row = self.layout.world + i
            place = []
            if spare_places and i < len(spare_places) and spare_places[i]:
                sp = spare_places[i]
                place = ["--daemon", sp["daemon"], "--store", sp["store"], "--node", sp["node"]]
            self._spawn(f"spare{i}-for{r}", base + ["--role", "spare", "--rank", str(r), "--row", str(row)]
                        + dev_args(row) + place + (["--resident"] if resident_spares else []), e)
        self.links: dict[int, Link] = {}
        deadline = time.monotonic() + start_timeout_s
        while len(self.links) < self.layout.world:
            self._check_started()
            try:
                link = self.carrier.wait_link(min(1.0, max(0.01, deadline - time.monotonic())))
            except TimeoutError:
                if time.monotonic() > deadline:
                    raise
                continue
            self.links[link.hello["rank"]] = link
        self.num_blocks = min(link.hello["num_blocks"] for link in self.links.values())
        self.epoch = 0
        self._boundary(0)
        self.changes: list[ChangeRecord] = []
        self.decode_steps_run = 0
        # host-side fault injection: (decode step, rank or ranks), or (prefill step, rank or ranks)
        self.kill_at_decode_step: tuple | None = None
        self.kill_at_prefill_step: tuple | None = None
        self.prefill_steps_run = 0
        self.notice_at_decode_step: tuple[int, int] | None = None  # (decode step, rank): a planned departure
        self.t_kill = self.t_kill_wall = 0.0
        self._finished: list[str] = []

    # ---- processes -------------------------------------------------------------------------------
    def _spawn(self, name: str, args: list[str], env: dict) -> None:
        out = subprocess.DEVNULL
        if self.log_dir:
            os.makedirs(self.log_dir, exist_ok=True)
            out = open(os.path.join(self.log_dir, f"{name}.log"), "w")  # noqa: SIM115
            self._logs.append(out)
        self.procs[name] = subprocess.Popen(args, env=env, stdout=out, stderr=subprocess.STDOUT)

    def _check_started(self) -> None:
        for name, p in self.procs.items():
            if p.poll() is not None and not name.startswith("spare"):
                raise RuntimeError(f"{name} exited with {p.returncode} during start-up")

    def pid_of(self, rank: int) -> int:
        return int(self.links[rank].hello["pid"])

    # ---- steps -----------------------------------------------------------------------------------
    FIRST_STEPS = 3  # steps timed after each resume (ChangeRecord.first_steps_ms)

    def execute(self, plan):
        t_step = time.monotonic()
        ids = self._execute(plan)
        if self.changes and len(self.changes[-1].first_steps_ms) < self.FIRST_STEPS and self.changes[-1].t_resumed:
            # the first steps after a change pay for whatever the change left cold (graphs,
            # mappings, caches): how long they take is part of what a client of the streams sees
            self.changes[-1].first_steps_ms.append(round((time.monotonic() - t_step) * 1e3, 3))
        return ids

    def _execute(self, plan):
        msg = {"op": "step", "epoch": self.epoch, "plan": plan}
        if self._finished:
            self._broadcast({"op": "finished", "ids": self._finished})
            self._finished = []
        victim = None
        if plan.is_prefill:
            self.prefill_steps_run += 1
            if self.kill_at_prefill_step and self.prefill_steps_run == self.kill_at_prefill_step[0]:
                victim = self.kill_at_prefill_step[1]
                self.kill_at_prefill_step = None
        if not plan.is_prefill:
            self.decode_steps_run += 1
            if self.kill_at_decode_step and self.decode_steps_run == self.kill_at_decode_step[0]:
                victim = self.kill_at_decode_step[1]
                self.kill_at_decode_step = None
            if self.notice_at_decode_step and self.decode_steps_run == self.notice_at_decode_step[0]:
                self.t_kill = time.monotonic()
                self.notice(self.notice_at_decode_step[1])
                self.notice_at_decode_step = None
        if victim is not None and not isinstance(victim, (list, tuple)):
            victim = [victim]
        if victim is not None and self.gpu:
            # on GPUs a rank leaves between steps (its kernels done), never mid-kernel
            msg = dict(msg, fail_at=plan.step, fail_rank=list(victim))
            self.t_kill, self.t_kill_wall = time.monotonic(), time.time()
            victim = None
        lost, errors = set(), {}
        for r, link in self.links.items():
            try:
                link.send(msg)
            except LinkClosed:
                lost.add(r)
        if victim is not None:
            self.t_kill, self.t_kill_wall = time.monotonic(), time.time()
            for v in victim:
                os.kill(self.pid_of(v), signal.SIGKILL)  # the fault: SIGKILL mid-step
        ids = None
        for r, link in self.links.items():
            if r in lost:
                continue
            try:
                while True:
                    reply = link.get(timeout=self.step_timeout_s, abandon=self._fault_pending)
                    if reply.get("step") == plan.step:
                        break
            except LinkClosed:
                lost.add(r)
                continue
            except StepAbandoned:
                # the coordinator's change for a fault is already under way: cut the step now
                raise RankLost(sorted(self.client.last_change.lost), "a membership change is pending") from None
            if reply["op"] == "error":
                errors[r] = reply["error"]
            elif "ids" in reply:
                ids = reply["ids"]
                self._logprobs = reply.get("logprobs")
        if lost or errors:
            raise RankLost(lost or set(errors), "; ".join(f"rank {r}: {e}" for r, e in errors.items()) or "link ended")
        return ids

    def _fault_pending(self) -> bool:
        """A change for a fault (not only planned departures) reached this head."""
        if self.client is None or not self.client.pending_change.is_set():
            return False
        ch = self.client.last_change
        return ch is not None and ch.epoch > self.epoch and not set(ch.lost) <= set(ch.departing)

    def fetch(self, ids):
        return ids

    def logprobs(self, n: int):
        """The last step's log-probability records (from the last stage's first column)."""
        return getattr(self, "_logprobs", None)

    def finished(self, req_id: str) -> None:
        self._finished.append(req_id)

    def decode_loop(self, plan, k):
        raise NotImplementedError("multi-step decode runs in one process; the multi-process engine steps singly")

    def _broadcast(self, msg: dict) -> None:
        for link in self.links.values():
            try:
                link.send(msg)
            except LinkClosed:
                pass

    def _boundary(self, epoch: int) -> dict[int, dict]:
        members = {}
        for r, link in self.links.items():
            if "row" in link.hello:
                self.rows[r] = int(link.hello["row"])
            members[r] = link.hello.get("key", str(r))
        # a pre-formed pipeline group is adopted only if every member holds it (two phases)
        adopt = False
        if self.layout.pipeline_parallel > 1 and any(not str(k).isdigit() for k in members.values()):
            for link in self.links.values():
                link.send({"op": "cover_query", "epoch": epoch, "members": members})
            have = []
            for link in self.links.values():
                while True:
                    reply = link.get(timeout=self.change_timeout_s)
                    if reply["op"] == "cover_have" and reply.get("epoch") == epoch:
                        break
                have.append(bool(reply["have"]))
            adopt = all(have)
        for link in self.links.values():
            link.send({"op": "boundary", "epoch": epoch, "rows": dict(self.rows), "members": members,
                       "adopt": adopt})
        self.adopted = {}
        computed = {}
        for r, link in self.links.items():
            while True:
                reply = link.get(timeout=self.change_timeout_s)
                if reply["op"] in ("ready", "error") and reply.get("epoch") == epoch:
                    break
            if reply["op"] == "error":
                raise RankLost({r}, f"boundary of epoch {epoch}: {reply['error']}")
            computed[r] = reply["computed"]
            self.adopted[r] = bool(reply.get("adopted"))
        # after the boundary every process is its rank in later plans
        for r, link in self.links.items():
            link.hello["key"] = str(r)
        return computed

    def _answer_replays(self) -> None:
        """Answer spares that a daemon launched with the engine's start-up record."""
        import json
        import queue

        while not self._closed:
            try:
                ask = self.client.replay_asks.get(timeout=0.5)
            except queue.Empty:
                continue
            row = None
            if self.region is not None:
                row = self._next_row
                self._next_row += 1
            rec = {"args": self._startup_args, "row": row, "gpu": self.gpu, "world": self.layout.world,
                   "token": self.token}
            try:
                self.client.offer_replay(ask, json.dumps(rec))
            except OSError:
                return

    # ---- membership change -----------------------------------------------------------------------
    def notice(self, rank: int, deadline_ms: int = 0) -> None:
        """Announce a planned departure of `rank` (drain): it finishes its step and leaves."""
        if self.client is None:
            raise EngineDown("no daemon link")
        self.client.notice(rank, deadline_ms or int(time.time() * 1000) + 30_000)

    def change_pending(self) -> bool:
        return self.client is not None and self.client.pending_change.is_set()

    def complete_change(self, engine, t_detect: float | None = None, cause: RankLost | None = None) -> ChangeRecord:
        """Wait for the coordinator's change and adopt it. `cause`: the loss this head saw in a
        step. A rank that answered with an error is alive, so nothing else reports it: the head
        reports it itself, unless a change for a fault is already under way; and a change that
        never comes ends in EngineDown naming the cause, not in a bare timeout."""
        if self.client is None:
            raise EngineDown("no daemon link: a lost rank cannot be replaced")
        t_detect = t_detect or time.monotonic()
        if cause is not None and cause.ranks and not self._fault_pending():
            try:
                self.client.report_lost(cause.ranks, f"step failed on the rank: {cause.detail}"[:512])
            except Exception:  # noqa: BLE001 - the wait below still bounds it
                pass
        try:
            h = self.client.wait_committed(timeout_s=self.change_timeout_s, after_epoch=self.epoch)
        except TimeoutError as e:
            raise EngineDown(f"no membership change within {self.change_timeout_s} s"
                             + (f" after {cause}" if cause is not None else "")) from e
        if h.kind == "abandoned":
            raise EngineDown(f"the coordinator abandoned epoch {h.epoch}: {h.detail}")
        mc = h.committed
        rec = ChangeRecord(mc.epoch, list(mc.lost), 0, t_detect, t_committed=time.monotonic(), t_fault=self.t_kill,
                           t_fault_wall=self.t_kill_wall if self.t_kill else 0.0)
        self.t_kill = 0.0
        rec.coordinator = {"reported_to_committed_ms": (mc.committed_at_us - mc.reported_at_us) / 1e3
                           if mc.reported_at_us else None, "pause_ms": mc.pause_ms,
                           # the coordinator's wall clock: comparable with time.time() on one host
                           "reported_at_us": mc.reported_at_us, "committed_at_us": mc.committed_at_us,
                           "delivered_at_us": mc.delivered_at_us, "acknowledged_at_us": mc.acknowledged_at_us,
                           "acks_at_us": {int(a.rank): int(a.received_at_us) for a in mc.acks}}
        lost = [r for r in mc.lost]
        ch = self.client.last_change
        planned = set(ch.departing) if ch is not None and ch.epoch == mc.epoch else set()
        departed = set()
        for r in lost:
            link = self.links.pop(r, None)
            if link is None:
                continue
            if r in planned and not link.closed.is_set():
                departed.add(r)
                try:  # a planned departure: it drains its commits and leaves
                    link.send({"op": "release"})
                    while link.get(timeout=self.change_timeout_s).get("op") != "released":
                        pass
                except (LinkClosed, TimeoutError):
                    pass
            link.close()
        for r in lost:
            offer = joinfmt.Offer(rank=r, epoch=mc.epoch, carrier=self.carrier.address, token=self.token,
                                  faulted=r not in departed)
            self.client.join(r, mc.epoch, joinfmt.encode(offer))
        for r in lost:
            link = self.carrier.wait_link(self.change_timeout_s, want=lambda hl, r=r: int(hl["rank"]) == r)
            self.links[r] = link
        rec.t_joined = time.monotonic()
        rec.outcome = 1 if lost else 0  # OUTCOME_REPLACE: a spare holds each lost rank
        self.links = dict(sorted(self.links.items()))
        computed = self._boundary(mc.epoch)
        rec.t_ready = time.monotonic()
        rec.coordinator["pre_formed_groups"] = sorted(r for r, a in self.adopted.items() if a)
        self.epoch = mc.epoch
        sch = engine.scheduler
        for req in sch.running:
            req.committed = min(int(c.get(req.req_id, 0)) for c in computed.values())
        rec.coordinator["committed_tokens"] = sorted({req.committed for req in sch.running})
        rec.coordinator["known_tokens"] = sorted({req.num_tokens for req in sch.running})
        sch.resume_from_committed()
        rec.t_resumed = time.monotonic()
        self.changes.append(rec)
        return rec

    def shutdown(self) -> None:
        self._closed = True
        for link in self.links.values():
            try:
                link.send({"op": "stop"})
            except LinkClosed:
                pass
        deadline = time.monotonic() + 30
        for p in self.procs.values():
            if p.poll() is None and not any(p.pid == int(link.hello["pid"]) for link in self.links.values()):
                p.terminate()
            try:
                p.wait(timeout=max(0.1, deadline - time.monotonic()))
            except subprocess.TimeoutExpired:
                p.kill()
                p.wait()
        if self.client is not None:
            self.client.close()
        self.carrier.close()
        if self.region is not None:
            self.region.close(unlink=True)
        for f in self._logs:
            f.close()


def failover(executor: MultiprocExecutor, engine):
    """The step wrapper: a step that loses a rank completes the membership change and retries."""

    def wrap(step_fn):
        def step():
            while True:
                try:
                    out = step_fn()
                except RankLost as e:
                    executor.complete_change(engine, t_detect=time.monotonic(), cause=e)
                    continue
                if executor.change_pending():  # a planned change: complete it at this boundary
                    executor.complete_change(engine, t_detect=time.monotonic())
                return out

        return step

    return wrap
