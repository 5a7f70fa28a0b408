"""A rank process of a multi-process engine: a worker, or a spare standing for a rank.

    python -m everserve_b200.serving.rank --role worker --rank 1 --engine e0 --model qwen2.5-0.5b \
        --tp 1 --pp 2 --head 127.0.0.1:PORT --rdzv 127.0.0.1:PORT --daemon unix:/run/n0.sock \
        --store unix:/run/store.sock [--device cpu] [--dtype float32] [--num-blocks N]
    python -m everserve_b200.serving.rank --role spare --rank 1 ...   # stands for rank 1

A worker builds its shard (stage layers, tensor column, paged KV cache), registers with its node's
daemon (``ROLE_WORKER``), links to the head and serves ops:

* ``step``: run the plan (receive the previous stage's output, forward, send to the next stage),
  then commit the step's KV rows and the requests' computed counts to the node's store
  (``MirrorCommittedKV``: a gather into a mapped staging file and a sender thread), fence the
  commit ``depth`` steps back, and reply (the last stage's column 0 with the sampled ids);
* ``boundary``: form the new epoch's groups (a rendezvous with every member of the epoch) and
  reply with what its cache holds (per-request computed counts);
* ``release``: a departing rank drains its commits and leaves (Goodbye, exit 0);
* ``stop``: leave.

A membership change reaches the rank through the daemon first (``Change``): the rank refuses its
live groups (so a send to a dead peer errors instead of waiting) unless only departures are
planned, and acks. The head then cuts the step and sends ``boundary``.

A spare builds the same shard ahead of time (weights, cache, a warm-up forward) and registers as
``ROLE_SPARE`` for its rank. When a ``Change`` names it in ``take``, it restores the lost rank's
committed KV from its node's store before it acks; the head's ``Join`` offer then tells it where to
link, it catches up on rows committed since its restore (a departing rank commits until the
boundary) and serves as the rank from then on.

Reference parity: the worker side of adapters/vllm/everserve_vllm/worker.py:1089-1266 (bootstrap,
boundary, resume, release_position) and the spare of spare_main.py / spare.py:96-281 (stand,
restore before the ack, join, catch-up).
"""

from __future__ import annotations

import argparse
import datetime
import os
import sys
import threading
import time

import torch
import torch.distributed as dist

from ..contract import join as joinfmt
from ..contract.daemon import DaemonConnection
from ..engine.config import EngineConfig
from ..engine.worker import Worker
from ..ops import dense
from ..proto import signals as sp
from ..runtime.groups import Exchange, GroupCollective, SwappableGroups
from ..runtime.layout import ParallelLayout
from ..runtime.runtime import Runtime
from ..state.kvcopy import PagedKV
from ..state.mirror import DEPTH, MirrorClient, MirrorCommittedKV
from .carrier import CarrierClient

_DTYPES = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}


def _store(addr: str, timeout_s: float = 60.0):
    host, _, port = addr.rpartition(":")
    return dist.TCPStore(host, int(port), is_master=False, timeout=datetime.timedelta(seconds=timeout_s))


def device_of(a: argparse.Namespace) -> torch.device:
    dev = torch.device(a.device)
    if dev.type == "cuda" and dev.index is None:
        dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    return dev


def config_of(a: argparse.Namespace) -> EngineConfig:
    """The engine configuration a rank process's arguments describe."""
    return EngineConfig(model=a.model, device=str(device_of(a)), dtype=_DTYPES[a.dtype], seed=a.seed,
                        block_size=a.block_size, num_blocks=a.num_blocks, max_batch=a.max_batch,
                        max_model_len=a.max_model_len, tensor_parallel=a.tp, pipeline_parallel=a.pp,
                        use_cuda_graphs=False, checkpoint=a.checkpoint)


class RankProcess:
    def __init__(self, a: argparse.Namespace, daemon_link=None):
        """`daemon_link`: the daemon connection of a spare that stood for any rank and was named
        to take `a.rank`; this process answers on it instead of registering again."""
        self.a = a
        self._link_device = daemon_link.device if daemon_link is not None else None
        self.engine = a.engine
        self.spare = a.role == "spare"
        self.rank = a.rank
        self.layout = ParallelLayout(a.tp, a.pp)
        dev = device_of(a)
        self.device = dev
        self.cfg = config_of(a)
        self.runtime = Runtime(self.rank)
        self.rdzv = _store(a.rdzv)
        from ..settings import load as load_settings

        self.groups = SwappableGroups(self.rdzv, self.rank, self.layout, dev, timeout_s=a.group_timeout,
                                      release_bound_s=load_settings().release_bound_ms / 1e3, on_leak=self._leaked)
        mc = self.cfg.model
        self.exchange = Exchange(self.groups, mc.hidden, self.cfg.dtype) if a.pp > 1 else None
        self.row = a.row if a.row is not None else self.rank
        self.rows = {r: r for r in range(self.layout.world)}  # rank position -> slot-region row
        self.region = None
        self.watch = None
        self._closing = threading.Event()
        coll = None
        if a.tp > 1 and dev.type == "cuda":
            coll = self._fused_collective(dev)
        elif a.tp > 1:
            coll = GroupCollective(self.groups)
        self.collective = coll
        t0 = time.monotonic()
        self.worker = None
        self.ckv = None
        self.host_weights = None
        if self.spare and a.resident and dev.type == "cuda":
            # a resident spare holds its shard in pinned host memory and no device memory while it
            # stands; the shard is copied to the device when it takes the rank
            self.host_weights = self._host_shard(coll)
        else:
            self._build_worker(coll)
        self.load_s = time.monotonic() - t0
        self.computed: dict[str, int] = {}
        self._commits: list[int] = []
        self.carrier: CarrierClient | None = None
        self.joined = threading.Event()
        self.offer: joinfmt.Offer | None = None
        self.leaving = False
        self.taken = False
        self.daemon = None
        self.cover = None
        self.key = f"R{self.rank}@{a.node}:{self.identity()[1]}" if self.spare else str(self.rank)
        if (a.daemon or daemon_link is not None) and a.pp > 1:
            from ..runtime.cover import Cover

            # each background formation gets its own store client (Cover's docstring)
            self.cover = Cover(lambda: _store(a.rdzv), self.key, self.engine, dev,
                               report=lambda r: self.daemon.report(r) if self.daemon is not None else None,
                               timeout_s=a.group_timeout)
        if daemon_link is not None:
            daemon_link.rank = self.rank
            daemon_link.participant = self
            self.daemon = daemon_link
        elif a.daemon:
            from ..contract.identity import identity

            pair = None
            cache_dir = os.environ.get("EVERSERVE_COMPILE_CACHE", "")
            if cache_dir and not self.spare:
                # the kernel build this worker loads, published for spares on nodes without it
                from ..contract.compile_cache import publish

                try:
                    pair = publish(cache_dir)
                except OSError as e:
                    self.runtime.trace("compile cache not published", why=str(e))
            self.daemon = DaemonConnection(a.daemon, self.engine, self, role=sp.ROLE_SPARE if self.spare else sp.ROLE_WORKER,
                                           stage=[self.layout.stage(self.rank)], node=a.node,
                                           identity=identity(self.cfg, self.engine), compile_cache=pair)

    def _build_worker(self, coll=None, weights=None) -> None:
        a, mc = self.a, self.cfg.model
        self.worker = Worker(self.cfg, rank=self.rank, collective=coll if coll is not None else self.collective,
                             pipe=self.exchange, device=str(self.device), weights=weights)
        self.caches = self.worker.runner.caches
        hkv = max(1, mc.kv_heads // a.tp)
        self.kv = PagedKV("heads_blocked", self.worker.num_blocks, a.block_size, hkv, mc.head_dim)
        if a.store:
            self.ckv = MirrorCommittedKV(MirrorClient(a.store), self.engine, self.rank, self.caches, self.kv,
                                         store_slots=self.worker.num_blocks * a.block_size)

    def _host_shard(self, coll) -> dict:
        """The rank's weights in pinned host memory (made on the device, then moved off it)."""
        w = Worker(self.cfg, rank=self.rank, collective=coll, pipe=self.exchange, device=str(self.device))
        host = {k: dense(t).to("cpu").pin_memory() for k, t in w.model.weights.items()}
        del w
        torch.cuda.empty_cache()
        return host

    # ---- the peer-memory tensor-parallel collective (GPUs) ----------------------------------------
    def _stage_rows(self) -> list[int]:
        stage = self.layout.stage(self.rank)
        ranks = [r for r in range(self.layout.world) if self.layout.stage(r) == stage]
        return [self.rows[r] for r in sorted(ranks, key=self.layout.column)]

    def _store_barrier(self, tag: str, rows: list[int], timeout_s: float = 60.0) -> None:
        self.rdzv.set(f"{tag}/{self.row}", b"1")
        self.rdzv.wait([f"{tag}/{r}" for r in rows], datetime.timedelta(seconds=timeout_s))

    def _fused_collective(self, dev):
        from ..parallel.fused import FusedTPCollective
        from ..parallel.slot import SlotRegion
        from ..runtime.slotwatch import SlotWatch
        from ..settings import load as load_settings

        self.settings = load_settings()
        self.region = SlotRegion.open(self.a.region)
        members = self._stage_rows()
        if self.spare:
            barrier = lambda: None  # noqa: E731 - a spare maps the members and waits for its take
        else:
            barrier = lambda: self._store_barrier("tp/e0", members)  # noqa: E731
        coll = FusedTPCollective(dev, region=self.region, row=self.row, members=members, barrier=barrier)
        # generous until the step period is measured (_sample_step), then `detect_steps` periods
        coll.set_bound_ns(self.settings.warmup_bound_ns())
        self._step_dt = []
        coll.set_beat_limit_us(int(self.settings.beat_limit_ms * 1000))
        if not self.spare:
            self._start_watch(coll, members)
            threading.Thread(target=self._premap_spares, args=(coll,), name="premap", daemon=True).start()
        return coll

    def _premap_spares(self, coll) -> None:
        """Map every standing spare's buffer ahead of a change, so the boundary only rewrites the
        member table (a non-member row's address is never read by the kernels)."""
        from ..parallel.slot import MAX_ROWS, OFF_PUBLISHED

        while not self._closing.is_set():
            for row in range(self.layout.world, MAX_ROWS):
                if row in coll._opened or not self.region.u32(row, OFF_PUBLISHED):
                    continue
                try:
                    coll.premap([row])
                except Exception as e:  # noqa: BLE001 - mapped at the boundary instead
                    self.runtime.trace("premap failed", row=row, why=str(e))
            self._closing.wait(0.5)

    def _start_watch(self, coll, members) -> None:
        from ..runtime.slotwatch import SlotWatch

        if self.watch is not None:
            self.watch.stop()

        def lost(ranks, why):
            coll.abort()  # the kernels waiting on the dead member leave now
            self.runtime.trace("slotwatch", ranks=ranks, why=why)
            if self.daemon is not None:
                try:
                    self.daemon.report_lost(ranks, f"slotwatch: {why}", reason=sp.REASON_FAULT)
                except OSError:
                    pass

        by_row = {row: r for r, row in self.rows.items()}
        self.watch = SlotWatch(self.region, self.row, lost, rank_of_row=lambda row: by_row.get(row, row),
                               members=members, poll_s=self.settings.poll_ms / 1e3,
                               hang_s=self.settings.hang_s, beat_limit_s=self.settings.beat_limit_ms / 1e3).start()

    def _leaked(self, release: str, seconds: float, total: int) -> None:
        """A refused group's release outlived its bound: tell the control plane, which retires this
        process by notice (a spare takes the rank at a later boundary)."""
        self.runtime.trace("release leaked", release=release, seconds=seconds, total=total)
        daemon = getattr(self, "daemon", None)
        if daemon is not None:
            try:
                daemon.report_leak(release, seconds, total)
            except OSError:
                pass

    # ---- participant (daemon reader thread) ------------------------------------------------------
    def identity(self) -> tuple[int, int]:
        if self._link_device is not None:  # the device the adopted link registered
            return self.rank, self._link_device
        if self.device.type == "cuda":
            return self.rank, self.device.index or 0
        # a CPU process has no device of its own: its row (one per process) stands in, so two
        # spares on one node are two seats
        return self.rank, self.row

    def on_change(self, change) -> str | None:
        self.runtime.trace("change", epoch=change.epoch)
        if self.cover is not None:
            self.cover.freeze()
        if self.spare and not self.taken:
            takes = [t for t in change.take if t.rank == self.rank]
            if not takes:
                return None
            try:
                if self.worker is None:  # a resident spare: its shard goes to the device now
                    t_copy = time.monotonic()
                    self._build_worker(weights=self.host_weights)
                    self.host_weights = None
                    self.runtime.trace("resident shard copied", seconds=time.monotonic() - t_copy)
                counts = self.ckv.restore(self.rank) if self.ckv is not None else {}
            except Exception as e:  # noqa: BLE001 - reported in the ack
                return f"restore failed: {e}"
            self.computed = dict(counts)
            self.taken = True
            self.runtime.stage_change(change)
            self.runtime.trace("restored", rows_step=self.ckv.restored_step if self.ckv else -1)
            return None
        self.runtime.stage_change(change)
        if self.rank in change.departing:
            self.leaving = True  # finish the step; the head releases this rank at the boundary
        elif not set(change.lost) <= set(change.departing):
            self.groups.refuse()
            if self.region is not None:
                self.collective.abort()
        return None

    def on_notice(self, rank: int, deadline_ms: int) -> None:
        self.runtime.trace("notice", rank=rank, deadline_ms=deadline_ms)

    def on_abandoned(self, epoch: int, detail: str) -> None:
        self.runtime.trace("abandoned", epoch=epoch, detail=detail)
        self.runtime.fault.set()

    def on_committed(self, committed) -> None:
        self.runtime.trace("committed", epoch=committed.epoch)

    def on_join(self, join) -> None:
        try:
            offer = joinfmt.decode(join.payload)
        except joinfmt.JoinFormatError as e:
            self.runtime.trace("join refused", why=str(e))
            return
        if isinstance(offer, joinfmt.Offer) and offer.rank == self.rank:
            self.offer = offer
            self.joined.set()

    def _column_keys(self, members: dict) -> list[str]:
        """This rank's column across the stages, in stage order, by the keys cover plans use."""
        rs = sorted((int(r) for r in members if self.layout.column(int(r)) == self.layout.column(self.rank)
                     and self.layout.replica(int(r)) == self.layout.replica(self.rank)))
        return [str(members[r] if r in members else members[str(r)]) for r in rs]

    def on_cover_plan(self, plan) -> None:
        if self.cover is not None:
            self.cover.apply(plan)

    def on_displaced(self, epoch: int, why: str) -> None:
        self.runtime.trace("displaced", epoch=epoch, why=why)

    # ---- serving ---------------------------------------------------------------------------------
    def warm(self) -> None:
        """One forward of a dummy step so the first real step pays no lazy set-up."""
        from ..engine.scheduler import ScheduledReq, StepPlan

        if self.layout.world > 1 or self.worker is None:
            return  # a lone forward of a middle stage has no peer; warm-up happens on the first step
        plan = StepPlan(0, False, [ScheduledReq("warm", [1], 0, [0], True)])
        self.worker.execute(plan)

    def link(self, address: str, token: str) -> None:
        hello = {"rank": self.rank, "row": self.row, "pid": os.getpid(), "role": "spare" if self.spare else "worker",
                 "token": token, "key": self.key,
                 "num_blocks": self.worker.num_blocks, "computed": dict(self.computed), "load_s": self.load_s}
        self.carrier = CarrierClient(address, hello)

    def serve(self) -> int:
        assert self.carrier is not None
        while True:
            try:
                msg = self.carrier.recv()
            except (ConnectionError, OSError, EOFError):
                return 1  # the head is gone
            op = msg["op"]
            if op == "step":
                self._step(msg)
            elif op == "boundary":
                self._boundary(msg)
            elif op == "cover_query":
                keys = self._column_keys(msg["members"])
                self.carrier.send({"op": "cover_have", "epoch": msg["epoch"], "rank": self.rank,
                                   "have": bool(self.cover is not None and self.cover.has(keys))})
            elif op == "finished":
                if self.ckv is not None and self.layout.stage(self.rank) == 0 and self.layout.column(self.rank) == 0:
                    for rid in msg["ids"]:
                        self.ckv.finished(rid)
                for rid in msg["ids"]:
                    self.computed.pop(rid, None)
            elif op == "release":
                self._drain()
                self.carrier.send({"op": "released", "rank": self.rank})
                if self.daemon is not None:
                    self.daemon.close(sp.STOP_CAUSE_STOPPED)
                return 0
            elif op == "stop":
                self._drain()
                if self.daemon is not None:
                    self.daemon.close(sp.STOP_CAUSE_STOPPED)
                return 0

    def _drain(self) -> None:
        if self.ckv is not None and self._commits:
            try:
                self.ckv.fence(self._commits[-1], timeout_s=30.0)
            except Exception:  # noqa: BLE001
                pass

    def _sample_step(self, seconds: float) -> None:
        """Fit the collective's wait bound to this rank's measured step period: every `step_sample`
        steps the median sets it to `detect_steps` periods (at least the floor)."""
        self._step_dt.append(seconds)
        n = max(1, self.settings.step_sample)
        if len(self._step_dt) >= n:
            period = sorted(self._step_dt)[len(self._step_dt) // 2]
            self.collective.set_bound_ns(self.settings.bound_ns(period))
            self._step_dt = []

    def _step(self, msg: dict) -> None:
        plan = msg["plan"]
        fail = msg.get("fail_rank")
        if msg.get("fail_at") == plan.step and (self.rank in fail if isinstance(fail, list) else self.rank == fail):
            # host-side fault injection: the process dies between steps, nothing of it in flight
            if self.device.type == "cuda":
                torch.cuda.synchronize(self.device)
            os.kill(os.getpid(), 9)
        try:
            if msg["epoch"] != self.runtime.epoch:
                raise RuntimeError(f"step of epoch {msg['epoch']} on a rank at epoch {self.runtime.epoch}")
            t_exec = time.monotonic()
            out = self.worker.execute(plan)
            if self.region is not None:
                if isinstance(out, torch.Tensor):
                    out = out.cpu()
                else:
                    torch.cuda.synchronize(self.device)
                self._sample_step(time.monotonic() - t_exec)
                st = self.collective.status() or self.worker.model.ops.check_status()
                if st:
                    raise RuntimeError(f"a collective of step {plan.step} failed (status {st}, late rows "
                                       f"{self.collective.late_rows()})")
            counts = {r.req_id: r.start_pos + len(r.token_ids) for r in plan.reqs}
            self.computed.update(counts)
            if self.ckv is not None:
                slots = [s for row in plan.slots(self.a.block_size) for s in row]
                self.ckv.commit(self.runtime.epoch, plan.step, counts, slots)
                self._commits.append(plan.step)
                if len(self._commits) > DEPTH:
                    self.ckv.fence(self._commits[-1 - DEPTH])
                del self._commits[:-(DEPTH + 1)]
            reply = {"op": "done", "step": plan.step, "rank": self.rank}
            if out is not None and self.layout.column(self.rank) == 0:
                reply["ids"] = out.tolist() if isinstance(out, torch.Tensor) else list(out)
                rows = self.worker.runner.logprob_rows(len(plan.reqs))
                if rows is not None:
                    reply["logprobs"] = rows
        except Exception as e:  # noqa: BLE001 - the head decides what a failed step means
            reply = {"op": "error", "step": plan.step, "rank": self.rank, "error": f"{type(e).__name__}: {e}"}
        self.carrier.send(reply)

    def _boundary(self, msg: dict) -> None:
        import faulthandler

        epoch = int(msg["epoch"])
        t0 = time.monotonic()
        # a boundary that takes longer than the group timeout leaves every thread's stack in the log
        faulthandler.dump_traceback_later(self.a.group_timeout + 15, exit=False)
        try:
            if self.spare and self.ckv is not None and self.ckv.restored_step >= 0:
                # rows the departing (or last) holder committed after the restore
                counts = self.ckv.restore(self.rank, since_step=self.ckv.restored_step + 1)
                self.computed.update(counts)
            pipe = None
            if self.cover is not None and msg.get("adopt"):
                pipe = self.cover.take(self._column_keys(msg["members"]))
                if pipe is None:
                    raise RuntimeError("the head chose a pre-formed group this rank does not hold")
            g = self.groups.form(epoch, self.rank, pipe=pipe)
            if self.cover is not None:
                self.cover.set_me(str(self.rank))
                self.cover.unfreeze()
            self.runtime.trace("groups", epoch=epoch, adopted=g.adopted)
            if "rows" in msg:
                self.rows = {int(r): int(row) for r, row in msg["rows"].items()}
            if self.region is not None:
                members = self._stage_rows()
                gone = [r for r in self.collective.members if r not in members]
                self.collective.set_members(members, epoch)
                self.collective.release_rows(gone)
                # a new member's first steps carry one-off costs: back to the warm-up bound, re-measured
                self.collective.set_bound_ns(self.settings.warmup_bound_ns())
                self._step_dt = []
                self.collective.resume()
                self._store_barrier(f"tp/e{epoch}", members)
                self._start_watch(self.collective, members)
            self.runtime.at_boundary(epoch)
            reply = {"op": "ready", "epoch": epoch, "rank": self.rank, "computed": dict(self.computed),
                     "form_s": time.monotonic() - t0, "adopted": g.adopted}
        except Exception as e:  # noqa: BLE001
            reply = {"op": "error", "epoch": epoch, "rank": self.rank, "error": f"{type(e).__name__}: {e}"}
        finally:
            faulthandler.cancel_dump_traceback_later()
        self.carrier.send(reply)

    def close(self) -> None:
        self._closing.set()
        if self.cover is not None:
            self.cover.close()
        if self.watch is not None:
            self.watch.stop()
        if self.ckv is not None:
            self.ckv.close()
        if self.region is not None:
            self.collective.close()


def parse(argv=None) -> argparse.Namespace:
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--role", choices=["worker", "spare"], default="worker")
    p.add_argument("--rank", type=int, required=True)
    p.add_argument("--engine", default="engine")
    p.add_argument("--model", default="qwen2.5-0.5b")
    p.add_argument("--tp", type=int, default=1)
    p.add_argument("--pp", type=int, default=1)
    p.add_argument("--device", default="cpu")
    p.add_argument("--dtype", default="float32", choices=list(_DTYPES))
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--block-size", type=int, default=16)
    p.add_argument("--num-blocks", type=int, default=None)
    p.add_argument("--max-batch", type=int, default=16)
    p.add_argument("--max-model-len", type=int, default=512)
    p.add_argument("--head", default="", help="the head's carrier address (workers)")
    p.add_argument("--rdzv", required=True, help="host:port of the engine's rendezvous store")
    p.add_argument("--daemon", default=os.environ.get("EVERSERVE_SOCKET", ""))
    p.add_argument("--store", default=os.environ.get("EVERSERVE_MIRROR_SOCKET", ""))
    p.add_argument("--node", default=os.environ.get("EVERSERVE_NODE", ""))
    p.add_argument("--group-timeout", type=float, default=30.0)
    p.add_argument("--region", default="", help="slot region name (GPU tensor parallelism)")
    p.add_argument("--row", type=int, default=None, help="this process's row in the slot region")
    p.add_argument("--threads", type=int, default=0)
    p.add_argument("--checkpoint", default=None, help="Hugging Face safetensors directory (default: random init)")
    p.add_argument("--resident", action="store_true",
                   help="a spare keeps its shard in pinned host memory until it takes a rank (GPUs)")
    return p.parse_args(argv)


def main(argv=None) -> int:
    import faulthandler
    import signal as _signal

    # `kill -USR1 <pid>` writes every thread's stack to this process's log (a hung rank is
    # inspected without stopping it)
    faulthandler.register(_signal.SIGUSR1, all_threads=True)
    a = parse(argv)
    if a.threads:
        torch.set_num_threads(a.threads)
    rp = RankProcess(a)
    try:
        if rp.spare:
            rp.warm()
            while not rp.joined.wait(0.1):
                pass
            assert rp.offer is not None
            rp.link(rp.offer.carrier, rp.offer.token)
        else:
            rp.link(a.head, os.environ.get("EVERSERVE_CARRIER_TOKEN", ""))
        return rp.serve()
    finally:
        rp.close()


if __name__ == "__main__":
    sys.exit(main())
