"""The head's links to its ranks: step plans down, results up.

One TCP connection per rank process, framed like every control-plane socket (4-byte big-endian
length + payload). The head listens on loopback or the node's address; a rank connects and says
``hello`` (JSON: its rank position, pid, the engine's carrier token). A hello without the token
is dropped before anything else is read, and only then do the two ends exchange pickled dicts
(``{"op": ...}``) between processes of one engine build. A link
that ends (the process died) or a reply carrying an error shows up as a lost rank to the head,
which then waits for the coordinator's membership change instead of guessing.

Reference parity: the executor <-> worker transport of
adapters/vllm/everserve_vllm/executor.py:660-853 (the response poll and the boundary messages);
here it is a plain socket per rank owned by the head.
"""

from __future__ import annotations

import json
import pickle
import queue
import socket
import threading
import time
from dataclasses import dataclass, field

from .. import wire


class LinkClosed(ConnectionError):
    pass


class StepAbandoned(RuntimeError):
    """The caller's `abandon` check said to stop waiting."""


def _send(sock: socket.socket, lock: threading.Lock, msg: dict) -> None:
    data = pickle.dumps(msg, protocol=pickle.HIGHEST_PROTOCOL)
    with lock:
        wire.send(sock, data)


def _recv(sock: socket.socket) -> dict:
    return pickle.loads(wire.recv(sock))


@dataclass
class Link:
    """The head's end of one rank's connection."""

    rank: int
    sock: socket.socket
    hello: dict
    inbox: queue.Queue = field(default_factory=queue.Queue)
    closed: threading.Event = field(default_factory=threading.Event)
    lock: threading.Lock = field(default_factory=threading.Lock)

    def send(self, msg: dict) -> None:
        if self.closed.is_set():
            raise LinkClosed(f"rank {self.rank}'s link is closed")
        try:
            _send(self.sock, self.lock, msg)
        except OSError as e:
            self.closed.set()
            raise LinkClosed(f"rank {self.rank}: {e}") from e

    def get(self, timeout: float | None = None, abandon=None) -> dict:
        """The next message; raises LinkClosed once the link ended and the inbox is empty, and
        StepAbandoned when `abandon()` turns true while waiting."""
        deadline = None if timeout is None else time.monotonic() + timeout
        while True:
            try:
                return self.inbox.get(timeout=0.002 if abandon is not None else 0.05)
            except queue.Empty:
                if self.closed.is_set() and self.inbox.empty():
                    raise LinkClosed(f"rank {self.rank}'s link ended") from None
                if abandon is not None and abandon():
                    raise StepAbandoned(f"stopped waiting for rank {self.rank}") from None
                if deadline is not None and time.monotonic() > deadline:
                    raise TimeoutError(f"rank {self.rank} sent nothing within {timeout} s") from None

    def close(self) -> None:
        self.closed.set()
        try:
            self.sock.shutdown(socket.SHUT_RDWR)
        except OSError:
            pass
        self.sock.close()


class CarrierServer:
    """The head's listener; links by rank position (a later hello for a rank replaces the link)."""

    def __init__(self, host: str = "127.0.0.1", port: int = 0, token: str = ""):
        self.token = token
        self.sock = socket.socket(socket.AF_INET, socket.SOCK_STREAM)
        self.sock.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
        self.sock.bind((host, port))
        self.sock.listen(64)
        self.address = f"{host}:{self.sock.getsockname()[1]}"
        self.links: dict[int, Link] = {}
        self.arrivals: queue.Queue[Link] = queue.Queue()
        self._unclaimed: list[Link] = []  # links that arrived while another was awaited
        self._stop = threading.Event()
        self._accept = threading.Thread(target=self._accept_loop, name="carrier-accept", daemon=True)
        self._accept.start()

    def _accept_loop(self) -> None:
        while not self._stop.is_set():
            try:
                s, _ = self.sock.accept()
            except OSError:
                return
            s.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
            threading.Thread(target=self._serve, args=(s,), daemon=True).start()

    def _serve(self, s: socket.socket) -> None:
        try:
            s.settimeout(10.0)
            hello = json.loads(wire.recv(s))
            s.settimeout(None)
        except (OSError, ConnectionError, ValueError, wire.FrameError):
            s.close()
            return
        if not isinstance(hello, dict) or hello.get("token", "") != self.token or "rank" not in hello:
            s.close()  # not one of this engine's ranks
            return
        link = Link(int(hello["rank"]), s, hello)
        self.arrivals.put(link)
        while True:
            try:
                link.inbox.put(_recv(s))
            except (OSError, ConnectionError, EOFError, pickle.UnpicklingError):
                link.closed.set()
                return

    def wait_link(self, timeout: float, want=None) -> Link:
        """The next arriving link (optionally one whose hello satisfies `want`). A link that
        arrives while another is wanted is kept for a later call (two spares taking two ranks
        link in either order)."""
        for i, link in enumerate(self._unclaimed):
            if want is None or want(link.hello):
                return self._unclaimed.pop(i)
        deadline = time.monotonic() + timeout
        while True:
            left = deadline - time.monotonic()
            if left <= 0:
                raise TimeoutError("no rank linked in time")
            try:
                link = self.arrivals.get(timeout=left)
            except queue.Empty:
                raise TimeoutError("no rank linked in time") from None
            if want is None or want(link.hello):
                return link
            self._unclaimed.append(link)

    def close(self) -> None:
        self._stop.set()
        try:
            self.sock.close()
        except OSError:
            pass
        for link in list(self.links.values()):
            link.close()


class CarrierClient:
    """A rank's end: connect, say hello, then receive ops and send replies."""

    def __init__(self, address: str, hello: dict, timeout_s: float = 30.0):
        self.sock = wire.connect(address, timeout=timeout_s)
        self.sock.settimeout(None)
        self.lock = threading.Lock()
        with self.lock:
            wire.send(self.sock, json.dumps(hello).encode())

    def recv(self) -> dict:
        return _recv(self.sock)

    def send(self, msg: dict) -> None:
        _send(self.sock, self.lock, msg)

    def close(self) -> None:
        try:
            self.sock.close()
        except OSError:
            pass
