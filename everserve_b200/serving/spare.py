"""A spare its node's daemon launched: fetch the engine's start-up record, then stand for a rank.

    (launched by everserve-node for a LaunchSpare; the environment names the engine, the rank it
     stands for, the device, the daemon's socket, the node and the store's socket)
    python -m everserve_b200.serving.spare

The spare does not know how the engine was started. It asks its daemon for the start-up record
(``ReplayAsk``; the daemon stamps where the answer must come back to and the coordinator relays
the ask to the engine's head), and the head answers with a ``ReplayOffer`` carrying the record as
JSON: the model and engine configuration, the rendezvous address, the slot region and a row of
it for this spare. With that the process builds the rank's shard, restores nothing yet, and
registers as ``ROLE_SPARE`` (``everserve_b200.serving.rank``); the daemon restarts it with a
backoff if it exits before it takes a rank.

A spare for any rank (``EVERSERVE_SPARE_RANK=any``: a policy slot without a rank, or a pool's
spare, ``EVERSERVE_ENGINES`` naming the pool's engines) holds no shard while it stands. It fetches
each engine's record, registers with each engine as a spare for any rank, and builds nothing until
a change names its node and device for a rank of one engine. Then it builds that rank (weights
loaded on notice), restores its committed KV, answers the change on the same link, and leaves the
other engines.

Reference parity: spare_main of adapters/vllm/everserve_vllm/spare_main.py:43-984 (policy and
discovery, replay fetch, stand per rank or for any position of a pool, register, wait for the
join) and the start-up record of replay.py:65-462 (here one JSON record instead of the engine
core's recorded broadcasts).
"""

from __future__ import annotations

import json
import os
import sys
import threading
import time

from ..contract.daemon import _Link
from ..proto import signals as sp


def fetch_startup(daemon: str, engine: str, rank: int, timeout_s: float = 120.0) -> dict:
    """Ask the engine's head for its start-up record; retries until the head answers."""
    deadline = time.monotonic() + timeout_s
    while True:
        link = _Link(daemon, timeout_s=min(10.0, timeout_s))
        try:
            link.send(sp.Signal(replay_ask=sp.ReplayAsk(engine=engine, rank=rank)))
            link.sock.settimeout(5.0)
            while True:
                sig = link.recv()
                if sig.WhichOneof("kind") == "replay_offer" and sig.replay_offer.engine == engine:
                    return json.loads(sig.replay_offer.handle)
        except (TimeoutError, OSError, ConnectionError):
            if time.monotonic() > deadline:
                raise TimeoutError(f"no start-up record from {engine}'s head within {timeout_s} s") from None
        finally:
            link.close()
        time.sleep(0.5)


def _rank_argv(rec: dict, rank: int, daemon: str) -> list[str]:
    argv = list(rec["args"]) + ["--role", "spare", "--rank", str(rank), "--daemon", daemon,
                                "--node", os.environ.get("EVERSERVE_NODE", "")]
    store = os.environ.get("EVERSERVE_MIRROR_SOCKET", "")
    if store:
        argv += ["--store", store]
    if rec.get("row") is not None:
        argv += ["--row", str(rec["row"])]
    if rec.get("gpu"):
        argv += ["--device", f"cuda:{os.environ.get('EVERSERVE_DEVICE', '0')}"]
    return argv


class AnyRankStand:
    """A spare for any rank of any of `engines` (module doc): one registration per engine."""

    def __init__(self, engines: list[str], daemon: str, timeout_s: float = 120.0):
        from ..contract.daemon import DaemonConnection
        from ..contract.identity import identity
        from .rank import config_of, parse

        self.daemon = daemon
        self.node = os.environ.get("EVERSERVE_NODE", "")
        self.device = int(os.environ.get("EVERSERVE_DEVICE", "0"))
        self.records = {e: fetch_startup(daemon, e, 0, timeout_s) for e in engines}
        if any(r.get("gpu") for r in self.records.values()):
            ensure_build(daemon, engines[0], 0)  # every rank of an engine loads the same build
        self.became = None  # the RankProcess it became
        self.error = ""
        self.done = threading.Event()
        self._lock = threading.Lock()
        self.links: dict[str, DaemonConnection] = {}
        for e in engines:
            a = parse(_rank_argv(self.records[e], 0, daemon))
            self.links[e] = DaemonConnection(daemon, e, _Seat(self, e), role=sp.ROLE_SPARE, any_rank=True,
                                             node=self.node, identity=identity(config_of(a), e))

    def take(self, engine: str, change) -> str | None:
        """A change names this node and device: become the rank, restore it, answer the change."""
        from .rank import RankProcess, parse

        mine = [t for t in change.take if t.node == self.node and t.device == self.device]
        if not mine:
            return None
        with self._lock:
            if self.became is not None:
                return f"this spare already took rank {self.became.rank} of {self.became.engine}"
            rank = int(mine[0].rank)
            try:
                rp = RankProcess(parse(_rank_argv(self.records[engine], rank, self.daemon)),
                                 daemon_link=self.links[engine])
            except Exception as e:  # noqa: BLE001 - reported in the ack
                self.error = f"building rank {rank}: {type(e).__name__}: {e}"
                self.done.set()
                return self.error
            self.became = rp
            for other, link in self.links.items():
                if other != engine:
                    link.close(sp.STOP_CAUSE_STOPPED)  # the other engines hear it leave
            err = rp.on_change(change)
            self.done.set()
            return err


class _Seat:
    """The participant of one engine's registration until the spare takes a rank."""

    def __init__(self, stand: AnyRankStand, engine: str):
        self.stand, self.engine = stand, engine

    def identity(self) -> tuple[int, int]:
        return 0, self.stand.device

    def on_change(self, change) -> str | None:
        return self.stand.take(self.engine, change)

    def on_notice(self, rank: int, deadline_ms: int) -> None:
        pass

    def on_abandoned(self, epoch: int, detail: str) -> None:
        pass

    def on_committed(self, committed) -> None:
        pass

    def on_join(self, join) -> None:
        pass

    def on_displaced(self, epoch: int, why: str) -> None:
        pass


def ensure_build(daemon: str, engine: str, rank: int) -> None:
    """A spare on a node without the kernel build (or told to fetch it) takes its rank's from the
    node's compile cache, fetched by the daemon from the stores that hold it."""
    from .. import _ext
    from ..contract import compile_cache

    cache_dir = os.environ.get("EVERSERVE_COMPILE_CACHE", "")
    if not cache_dir or (_ext.available() and os.environ.get("EVERSERVE_FETCH_COMPILE_CACHE") != "1"):
        return
    ready = compile_cache.want(daemon, engine, rank)
    compile_cache.load_from_cache(cache_dir, ready)


def main() -> int:
    daemon = os.environ["EVERSERVE_SOCKET"]
    rank_s = os.environ.get("EVERSERVE_SPARE_RANK", "any")
    engines = [e for e in os.environ.get("EVERSERVE_ENGINES", "").split(",") if e] or [os.environ["EVERSERVE_ENGINE"]]
    from .rank import main as rank_main

    if rank_s.isdigit():
        rank = int(rank_s)
        rec = fetch_startup(daemon, engines[0], rank)
        if rec.get("gpu"):
            ensure_build(daemon, engines[0], rank)
        return rank_main(_rank_argv(rec, rank, daemon))
    stand = AnyRankStand(engines, daemon)
    stand.done.wait()
    rp = stand.became
    if rp is None:
        print(stand.error, file=sys.stderr)
        return 1
    try:
        while not rp.joined.wait(0.1):
            pass
        assert rp.offer is not None
        rp.link(rp.offer.carrier, rp.offer.token)
        return rp.serve()
    finally:
        rp.close()


if __name__ == "__main__":
    sys.exit(main())
