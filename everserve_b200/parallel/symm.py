"""Symmetric peer buffers on driver VMM allocations, shared by file descriptor.

Each member creates its buffer with ``vmm_create`` (an exportable physical allocation mapped on its
own device) and serves the exported descriptor on a Unix socket next to the slot region
(``<region>.r<row>.fd``; ``SCM_RIGHTS`` passes the descriptor). A member that needs a peer's
buffer connects, receives the descriptor and maps it with access for its own device
(``vmm_import``: a peer mapping over NVLink). The descriptor is closed right after the import.

The physical memory of a buffer lives until every process has released its mapping, so a member
that dies leaves its buffer valid for the survivors: a kernel still pushing words to it, or
polling words in it, touches live memory and leaves through its bounded wait. This is why the
failure-detecting collectives use these buffers instead of legacy CUDA IPC, whose exporter frees
the memory under its importers when it exits.
"""

from __future__ import annotations

import os
import socket
import time
import threading


class SymmetricBuffer:
    def __init__(self, C, nbytes: int, sock_path: str):
        self.C = C
        self.ptr, self.size, self.handle, self.fd = (int(v) for v in C.vmm_create(nbytes))
        self.sock_path = sock_path
        try:
            os.unlink(sock_path)
        except FileNotFoundError:
            pass
        self._srv = socket.socket(socket.AF_UNIX, socket.SOCK_STREAM)
        self._srv.bind(sock_path)
        self._srv.listen(16)
        self._stop = threading.Event()
        self._t = threading.Thread(target=self._serve, name="symm-fd", daemon=True)
        self._t.start()

    def _serve(self) -> None:
        while not self._stop.is_set():
            try:
                c, _ = self._srv.accept()
            except OSError:
                return
            try:
                socket.send_fds(c, [self.size.to_bytes(8, "little")], [self.fd])
            except OSError:
                pass
            finally:
                c.close()

    def close(self) -> None:
        self._stop.set()
        try:
            self._srv.close()
        except OSError:
            pass
        try:
            os.unlink(self.sock_path)
        except FileNotFoundError:
            pass
        if self.ptr:
            self.C.vmm_release(self.ptr, self.size, self.handle, self.fd)
            self.ptr = 0


class PeerMapping:
    """A peer's buffer mapped into this process (released explicitly, never by the peer's exit)."""

    def __init__(self, C, sock_path: str, timeout_s: float = 30.0):
        self.C = C
        # the peer may still be creating its buffer (loading weights, say): its socket appears
        # when it is ready, so a missing or refusing socket is retried until the timeout
        deadline = time.monotonic() + timeout_s
        while True:
            s = socket.socket(socket.AF_UNIX, socket.SOCK_STREAM)
            s.settimeout(timeout_s)
            try:
                s.connect(sock_path)
                msg, fds, _, _ = socket.recv_fds(s, 8, 1)
                break
            except (FileNotFoundError, ConnectionRefusedError):
                if time.monotonic() > deadline:
                    raise
                time.sleep(0.01)
            finally:
                s.close()
        if not fds or len(msg) != 8:
            raise RuntimeError(f"no buffer descriptor from {sock_path}")
        size = int.from_bytes(msg, "little")
        try:
            self.ptr, self.size, self.handle = (int(v) for v in C.vmm_import(fds[0], size))
        finally:
            os.close(fds[0])

    def close(self) -> None:
        if self.ptr:
            self.C.vmm_release(self.ptr, self.size, self.handle, -1)
            self.ptr = 0
