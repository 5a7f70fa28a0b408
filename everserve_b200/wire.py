"""Frames on the control-plane sockets: a 4-byte big-endian payload length, then the payload.

Frames above ``MAX_FRAME`` (16 MiB) are refused on both sides. Reference parity: the frame codec of
core/everserve/wire.py:15-79 and wire/src/frame.rs:9-61 (same format, so any member speaks to
the C++ daemon and store).
"""

from __future__ import annotations

import socket
import struct

MAX_FRAME = 16 << 20


class FrameError(RuntimeError):
    pass


def encode(payload: bytes) -> bytes:
    if len(payload) > MAX_FRAME:
        raise FrameError(f"frame of {len(payload)} bytes above the {MAX_FRAME} cap")
    return struct.pack(">I", len(payload)) + payload


def _recv_exact(sock: socket.socket, n: int) -> bytes:
    buf = bytearray()
    while len(buf) < n:
        chunk = sock.recv(n - len(buf))
        if not chunk:
            raise ConnectionError("peer closed the connection")
        buf += chunk
    return bytes(buf)


def send(sock: socket.socket, payload: bytes) -> None:
    sock.sendall(encode(payload))


def recv(sock: socket.socket) -> bytes:
    (n,) = struct.unpack(">I", _recv_exact(sock, 4))
    if n > MAX_FRAME:
        raise FrameError(f"incoming frame of {n} bytes above the cap")
    return _recv_exact(sock, n)


class FrameBuffer:
    """Accumulates bytes and yields complete frames (for non-blocking readers)."""

    def __init__(self):
        self._buf = bytearray()

    def feed(self, data: bytes) -> list[bytes]:
        self._buf += data
        out = []
        while len(self._buf) >= 4:
            (n,) = struct.unpack_from(">I", self._buf, 0)
            if n > MAX_FRAME:
                raise FrameError(f"incoming frame of {n} bytes above the cap")
            if len(self._buf) < 4 + n:
                break
            out.append(bytes(self._buf[4 : 4 + n]))
            del self._buf[: 4 + n]
        return out


def parse_address(addr: str) -> tuple[int, object]:
    """``unix:/path`` or an absolute path -> (AF_UNIX, path); ``host:port`` -> (AF_INET, (host, port))."""
    if addr.startswith("unix:"):
        return socket.AF_UNIX, addr[5:]
    if addr.startswith("/"):
        return socket.AF_UNIX, addr
    host, _, port = addr.rpartition(":")
    return socket.AF_INET, (host or "127.0.0.1", int(port))


def connect(addr: str, timeout: float = 10.0) -> socket.socket:
    fam, target = parse_address(addr)
    s = socket.socket(fam, socket.SOCK_STREAM)
    s.settimeout(timeout)
    s.connect(target)
    if fam == socket.AF_INET:
        s.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
    return s
