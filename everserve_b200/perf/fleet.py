"""Control-plane scale: one coordinator and a fleet of simulated node daemons.

    python -m everserve_b200.perf.fleet [--nodes 256] [--gpus 8] [--losses 20]

The real ``everserve-coord`` links to N simulated daemons, each speaking coord.proto over the
coordinator's socket from one asyncio process: a hello with its GPUs, heartbeats every 500 ms, and
the registrations of its processes. Every engine is TP``gpus`` on one node; every ninth node is a
spare node whose GPUs hold a spare for any rank of one engine each. Losses are reported one at a
time (a rank of a random engine); the simulated daemons answer every delivery at once with their
named ranks' acks, so what is measured is the coordinator: from the loss report to the commit
(its own stamps, ``committed_at_us - reported_at_us``) and the round trip the reporting daemon
sees. It prints one JSON line with p50 / p99 / max of both, and the time until the coordinator has
taken in the whole fleet's hellos and registrations.

Reference parity: the synthetic fleets of fake daemons the reference measures its control plane
with (bench/runs cell-s1, up to 5,000 daemons); the simulated daemon here is this framework's.
"""

from __future__ import annotations

import argparse
import asyncio
import json
import os
import random
import shutil
import struct
import subprocess
import tempfile
import time


def _pct(xs, q):
    xs = sorted(xs)
    if not xs:
        return None
    return round(xs[min(len(xs) - 1, max(0, int(round(q / 100 * (len(xs) - 1)))))], 3)


class SimNode:
    """One simulated daemon: links, registers its processes, acks what it is delivered."""

    def __init__(self, name: str, gpus: int, workers: dict[str, list[int]], spares: list[tuple[str, int]]):
        self.name, self.gpus = name, gpus
        self.workers = workers  # engine -> ranks on this node (device = rank)
        self.spares = spares  # (engine, device) any-rank spares
        self.committed: dict[str, asyncio.Future] = {}
        self.writer = None

    async def send(self, msg) -> None:
        data = msg.SerializeToString()
        self.writer.write(struct.pack(">I", len(data)) + data)
        await self.writer.drain()

    async def run(self, path: str, ready: asyncio.Event, linked: list) -> None:
        from ..proto import coord as cp
        from ..proto import signals as sp

        delay = 0.05
        while True:  # as a daemon does: a link refused is tried again with backoff
            try:
                reader, self.writer = await asyncio.open_unix_connection(path)
                break
            except OSError:
                await asyncio.sleep(delay)
                delay = min(delay * 2, 1.0)
        hello = cp.DaemonToCoord(hello=cp.DaemonHello(node=self.name, heartbeat_ms=500, protocol=sp.PROTOCOL_VERSION,
                                                      devices=[cp.Device(index=i, uuid=f"GPU-{self.name}-{i}",
                                                                         **{"class": "NVIDIA B200"},
                                                                         memory_bytes=183359 << 20)
                                                               for i in range(self.gpus)]))
        await self.send(hello)
        for eng, ranks in self.workers.items():
            for r in ranks:
                await self.send(cp.DaemonToCoord(worker_event=cp.WorkerEvent(
                    engine=eng, kind=cp.WorkerEvent.WORKER_REGISTERED, rank=r, world_size=self.gpus, device=r,
                    pid=1000 + r)))
        for eng, dev in self.spares:
            await self.send(cp.DaemonToCoord(worker_event=cp.WorkerEvent(
                engine=eng, kind=cp.WorkerEvent.SPARE_REGISTERED, any_rank=True, device=dev, pid=2000 + dev)))
        linked.append(time.monotonic())
        ready.set()
        asyncio.get_running_loop().create_task(self._heartbeats())
        while True:
            head = await reader.readexactly(4)
            msg = cp.CoordToDaemon()
            msg.ParseFromString(await reader.readexactly(struct.unpack(">I", head)[0]))
            kind = msg.WhichOneof("kind")
            if kind == "deliver":
                d = msg.deliver
                acks = [sp.Ack(rank=r, epoch=d.change.epoch) for r in list(d.to_ranks) + list(d.to_spares)]
                await self.send(cp.DaemonToCoord(delivered=cp.Delivered(request_id=d.request_id, engine=d.engine,
                                                                        epoch=d.change.epoch, acks=acks)))
            elif kind == "committed":
                f = self.committed.pop(msg.committed.engine, None)
                if f is not None and not f.done():
                    f.set_result(msg.committed)

    async def _heartbeats(self) -> None:
        from ..proto import coord as cp

        while True:
            await asyncio.sleep(0.5)
            await self.send(cp.DaemonToCoord(heartbeat=cp.Heartbeat()))

    async def lose(self, engine: str, rank: int):
        from ..proto import coord as cp
        from ..proto import signals as sp

        f = asyncio.get_running_loop().create_future()
        self.committed[engine] = f
        t0 = time.monotonic()
        await self.send(cp.DaemonToCoord(lost_report=cp.LostReport(engine=engine, lost=sp.RankLost(
            ranks=[rank], reason=sp.REASON_FAULT, detail="simulated"))))
        c = await asyncio.wait_for(f, timeout=30)
        return c, (time.monotonic() - t0) * 1e3


def _get(api: str, path: str) -> dict:
    import http.client

    host, _, port = api.rpartition(":")
    c = http.client.HTTPConnection(host, int(port), timeout=10)
    try:
        c.request("GET", path)
        return json.loads(c.getresponse().read())
    finally:
        c.close()


async def _spare_standing(api: str, engine: str, timeout_s: float = 120.0) -> float:
    """Wait until the coordinator admitted `engine`'s spare; returns how long that took."""
    t0 = time.monotonic()
    while time.monotonic() - t0 < timeout_s:
        try:
            view = await asyncio.to_thread(_get, api, f"/v1/engines/{engine}")
            if view["status"]["spares"]:
                return time.monotonic() - t0
        except (OSError, ValueError, KeyError):
            pass
        await asyncio.sleep(0.05)
    raise TimeoutError(f"{engine}'s spare was not admitted within {timeout_s} s")


async def run_fleet(coord_bin: str, nodes: int, gpus: int, losses: int, seed: int = 0) -> dict:
    from ..serving.cluster import free_port

    work = tempfile.mkdtemp(prefix="es-fleet-")
    sock = os.path.join(work, "coord.sock")
    api = f"127.0.0.1:{free_port()}"
    log = open(os.path.join(work, "coord.log"), "w")  # noqa: SIM115
    proc = subprocess.Popen([coord_bin, "--listen", f"unix:{sock}", "--spec-store", os.path.join(work, "spec"),
                             "--node-loss-misses", "20", "--api-addr", api], stdout=log, stderr=subprocess.STDOUT)
    try:
        for _ in range(200):
            if os.path.exists(sock):
                break
            await asyncio.sleep(0.05)
        sims, engines = [], []
        spare_nodes = [i for i in range(nodes) if i % 9 == 8]
        serving = [i for i in range(nodes) if i % 9 != 8]
        for i in serving:
            engines.append(f"e{i}")
        for i in range(nodes):
            if i in spare_nodes:
                k = spare_nodes.index(i)
                mine = engines[k * gpus:(k + 1) * gpus]
                sims.append(SimNode(f"n{i}", gpus, {}, [(e, d) for d, e in enumerate(mine)]))
            else:
                sims.append(SimNode(f"n{i}", gpus, {f"e{i}": list(range(gpus))}, []))
        linked: list[float] = []
        t0 = time.monotonic()
        readies = []
        for s in sims:
            ev = asyncio.Event()
            readies.append(ev)
            asyncio.get_running_loop().create_task(s.run(sock, ev, linked))
        await asyncio.gather(*(e.wait() for e in readies))
        rng = random.Random(seed)
        covered = [e for k in range(len(spare_nodes)) for e in engines[k * gpus:(k + 1) * gpus]]
        # the fleet is up once the coordinator took in the last registrations sent
        await _spare_standing(api, covered[-1])
        link_up_s = time.monotonic() - t0
        coord_ms, rtt_ms = [], []
        for e in rng.sample(covered, min(losses, len(covered))):
            node = sims[int(e[1:])]
            await _spare_standing(api, e)
            c, rtt = await node.lose(e, rng.randrange(gpus))
            m = c.membership
            coord_ms.append((m.committed_at_us - m.reported_at_us) / 1e3)
            rtt_ms.append(rtt)
        return {"metric": "control-plane change latency at fleet scale", "nodes": nodes, "gpus_per_node": gpus,
                "engines": len(engines), "losses": len(coord_ms), "link_up_s": round(link_up_s, 3),
                "report_to_commit_ms": {"p50": _pct(coord_ms, 50), "p99": _pct(coord_ms, 99),
                                        "max": round(max(coord_ms), 3) if coord_ms else None},
                "daemon_round_trip_ms": {"p50": _pct(rtt_ms, 50), "p99": _pct(rtt_ms, 99),
                                         "max": round(max(rtt_ms), 3) if rtt_ms else None}}
    finally:
        proc.terminate()
        try:
            proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            proc.kill()
        log.close()
        if os.environ.get("ES_FLEET_KEEP"):
            print("kept", work)
        else:
            shutil.rmtree(work, ignore_errors=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--nodes", type=int, default=256)
    ap.add_argument("--gpus", type=int, default=8)
    ap.add_argument("--losses", type=int, default=20)
    ap.add_argument("--seed", type=int, default=0)
    a = ap.parse_args()
    from ..serving.cluster import binary

    print(json.dumps(asyncio.run(run_fleet(binary("everserve-coord"), a.nodes, a.gpus, a.losses, a.seed))))


if __name__ == "__main__":
    main()
