"""The reference tier's fault channel: a process learns of a fault on the host, never on a device.

``FaultListener`` accepts connections on a local address and queues the fault messages it
receives; ``FaultClient`` sends one; ``broadcast_fault`` sends one to every listener that is
still there (a listener of a dead process is skipped).

Reference parity: core/everserve/reference/control.py:26-158.
"""

from __future__ import annotations

import queue
import threading
from multiprocessing.connection import Client, Listener

AUTH = b"everserve-fault"


class FaultListener:
    def __init__(self, address=("127.0.0.1", 0)):
        self._l = Listener(address, authkey=AUTH)
        self.address = self._l.address
        self.faults: queue.Queue = queue.Queue()
        threading.Thread(target=self._accept, daemon=True).start()

    def _accept(self) -> None:
        while True:
            try:
                c = self._l.accept()
            except OSError:
                return
            try:
                self.faults.put(c.recv())
            except (EOFError, OSError):
                pass
            finally:
                c.close()

    def next(self, timeout: float | None = None):
        return self.faults.get(timeout=timeout)

    def close(self) -> None:
        self._l.close()


class FaultClient:
    def __init__(self, address):
        self.address = address

    def send(self, fault) -> bool:
        try:
            c = Client(self.address, authkey=AUTH)
        except OSError:
            return False
        try:
            c.send(fault)
        finally:
            c.close()
        return True


def broadcast_fault(addresses, fault) -> list:
    """Send `fault` to every listener; returns the addresses that took it."""
    return [a for a in addresses if FaultClient(a).send(fault)]
