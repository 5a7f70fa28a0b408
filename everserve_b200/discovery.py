"""Where a node's daemon and store listen: records in a discovery directory, or the environment.

A daemon started with ``--discovery-dir DIR`` writes ``DIR/<node>.json`` (``DaemonRecord`` in proto3
JSON: node, address, engines, start time, pid, store address, host). Processes find their node's
daemon through ``local_daemon(node)``: the environment (``EVERSERVE_DAEMON_SOCKET``,
``EVERSERVE_MIRROR_SOCKET``, ``EVERSERVE_HOST_IP``) first, then the directory.

Reference parity: core/everserve/discovery.py:21-140 (file backend, same record, same variables).
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from pathlib import Path

from google.protobuf import json_format

from .proto import discovery as dp

DAEMON_SOCKET_ENV = "EVERSERVE_DAEMON_SOCKET"
MIRROR_SOCKET_ENV = "EVERSERVE_MIRROR_SOCKET"
HOST_IP_ENV = "EVERSERVE_HOST_IP"
DISCOVERY_DIR_ENV = "EVERSERVE_DISCOVERY_DIR"


@dataclass(frozen=True)
class DaemonRecord:
    node: str
    address: str
    engines: tuple[str, ...] = ()
    started_at_ms: int = 0
    pid: int = 0
    mirror_address: str = ""
    host_ip: str = ""

    @property
    def host(self) -> str:
        return self.host_ip or "127.0.0.1"

    @classmethod
    def from_message(cls, m) -> "DaemonRecord":
        return cls(m.node, m.address, tuple(m.engines), m.started_at_ms, m.pid, m.mirror_address, m.host)

    def to_message(self):
        return dp.DaemonRecord(node=self.node, address=self.address, engines=list(self.engines),
                               started_at_ms=self.started_at_ms, pid=self.pid, mirror_address=self.mirror_address,
                               host=self.host_ip)


class FileDiscovery:
    def __init__(self, directory: str | Path):
        self.dir = Path(directory)

    def daemons(self) -> list[DaemonRecord]:
        out = []
        if not self.dir.is_dir():
            return out
        for p in sorted(self.dir.glob("*.json")):
            try:
                out.append(DaemonRecord.from_message(json_format.Parse(p.read_text(), dp.DaemonRecord())))
            except (OSError, json_format.ParseError):
                continue
        return out

    def daemon(self, node: str) -> DaemonRecord | None:
        return next((d for d in self.daemons() if d.node == node), None)

    def publish(self, rec: DaemonRecord) -> None:
        self.dir.mkdir(parents=True, exist_ok=True)
        tmp = self.dir / f".{rec.node}.json.tmp"
        tmp.write_text(json_format.MessageToJson(rec.to_message()))
        os.replace(tmp, self.dir / f"{rec.node}.json")


def local_daemon(node: str, discovery_dir: str | Path | None = None) -> DaemonRecord | None:
    sock = os.environ.get(DAEMON_SOCKET_ENV)
    if sock:
        return DaemonRecord(node, sock, mirror_address=os.environ.get(MIRROR_SOCKET_ENV, ""),
                            host_ip=os.environ.get(HOST_IP_ENV, ""))
    d = discovery_dir or os.environ.get(DISCOVERY_DIR_ENV)
    return FileDiscovery(d).daemon(node) if d else None
