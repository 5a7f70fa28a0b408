"""The slot region: a node-local shared-memory file every member of a group maps.

It carries, per member row (up to 8: seven ranks and a spare), the control words the collective
kernels read and write through a device mapping of pinned host memory, and the words the executor,
the watchdog and the members exchange on the host:

    row r at ROW0 + r * ROW_BYTES:
      +0   abort    u32  host -> device: non-zero makes a kernel waiting on peers leave
      +4   late     u32  device -> host: rows a wait has waited for past `bound` (a bit mask)
      +8   bound_ns u64  host -> device: wait after which late members are named (0: off)
      +16  status   u32  device -> host: last failure of a collective (1 timeout, 2 aborted, 4 dead)
      +20  beat     u32  the member's process: heartbeat counter (a native thread, ~0.5 ms)
      +24  beat_limit_us u32 host -> device: a peer's beat standing still this long is a death
      +32  pid      i64  the member's process
      +40  step     i64  the step in flight (0: idle) -- the step word the watchdog reads
      +48  lost     u32  set by a watcher that found the member dead
      +52  published u32 the IPC handle below is valid
      +64  order    i32[9] member count, then rows in member (rank) order, as this member sees it
      +128 handle   64 bytes: CUDA IPC handle of the member's symmetric buffer
    header at 0: magic, version, rows

Reference parity: the region of core/everserve/comm/slotkernel.py:71-120,293-576 (ctrl words,
published handles, late mask, bound, pid, lost, step). The byte layout here is this framework's.
"""

from __future__ import annotations

import mmap
import os
import struct
import time

MAGIC = b"ESB2SLOT"
VERSION = 1
MAX_ROWS = 8
ROW0 = 4096
ROW_BYTES = 256
SIZE = 8192

OFF_ABORT, OFF_LATE, OFF_BOUND, OFF_STATUS, OFF_BEAT, OFF_BEAT_LIMIT = 0, 4, 8, 16, 20, 24
OFF_PID, OFF_STEP, OFF_LOST, OFF_PUBLISHED = 32, 40, 48, 52
OFF_ORDER, OFF_HANDLE = 64, 128
HANDLE_BYTES = 64


def shm_dir() -> str:
    return os.environ.get("EVERSERVE_SHM_DIR", "/dev/shm")


class SlotRegion:
    def __init__(self, path: str, create: bool = False):
        self.path = path
        if create:
            fd = os.open(path, os.O_RDWR | os.O_CREAT | os.O_TRUNC, 0o660)
            os.ftruncate(fd, SIZE)
        else:
            fd = os.open(path, os.O_RDWR)
        try:
            self.mm = mmap.mmap(fd, SIZE)
        finally:
            os.close(fd)
        if create:
            self.mm[:SIZE] = bytes(SIZE)
            self.mm[0:8] = MAGIC
            struct.pack_into("<II", self.mm, 8, VERSION, MAX_ROWS)
        elif bytes(self.mm[0:8]) != MAGIC:
            raise ValueError(f"{path} is not a slot region")
        self._dev_base = 0
        self._registered = False

    @classmethod
    def create(cls, name: str) -> "SlotRegion":
        return cls(os.path.join(shm_dir(), name), create=True)

    @classmethod
    def open(cls, name: str, timeout_s: float = 60.0) -> "SlotRegion":
        path = os.path.join(shm_dir(), name)
        t0 = time.monotonic()
        while not os.path.exists(path):
            if time.monotonic() - t0 > timeout_s:
                raise TimeoutError(f"slot region {path} did not appear")
            time.sleep(0.01)
        return cls(path)

    # ---- words ---------------------------------------------------------------------------------
    def _off(self, row: int, field: int) -> int:
        if not 0 <= row < MAX_ROWS:
            raise ValueError(f"row {row} out of range")
        return ROW0 + row * ROW_BYTES + field

    def u32(self, row: int, field: int) -> int:
        return struct.unpack_from("<I", self.mm, self._off(row, field))[0]

    def set_u32(self, row: int, field: int, v: int) -> None:
        struct.pack_into("<I", self.mm, self._off(row, field), v & 0xFFFFFFFF)

    def i64(self, row: int, field: int) -> int:
        return struct.unpack_from("<q", self.mm, self._off(row, field))[0]

    def set_i64(self, row: int, field: int, v: int) -> None:
        struct.pack_into("<q", self.mm, self._off(row, field), v)

    def abort(self, row: int) -> int:
        return self.u32(row, OFF_ABORT)

    def set_abort(self, rows, value: int = 1) -> None:
        for r in rows:
            self.set_u32(r, OFF_ABORT, value)

    def late(self, row: int) -> int:
        return self.u32(row, OFF_LATE)

    def clear_late(self, row: int) -> None:
        self.set_u32(row, OFF_LATE, 0)

    def set_bound_ns(self, rows, ns: int) -> None:
        for r in rows:
            struct.pack_into("<Q", self.mm, self._off(r, OFF_BOUND), int(ns))

    def bound_ns(self, row: int) -> int:
        return struct.unpack_from("<Q", self.mm, self._off(row, OFF_BOUND))[0]

    def status(self, row: int) -> int:
        return self.u32(row, OFF_STATUS)

    def beat(self, row: int) -> int:
        return self.u32(row, OFF_BEAT)

    def beat_address(self, row: int) -> int:
        """Host address of the row's beat word (what the native heartbeat thread advances)."""
        import ctypes

        return ctypes.addressof(ctypes.c_char.from_buffer(self.mm)) + self._off(row, OFF_BEAT)

    def set_beat_limit_us(self, rows, us: int) -> None:
        for r in rows:
            self.set_u32(r, OFF_BEAT_LIMIT, us)

    def set_pid(self, row: int, pid: int) -> None:
        self.set_i64(row, OFF_PID, pid)

    def pid(self, row: int) -> int:
        return self.i64(row, OFF_PID)

    def set_step(self, row: int, step: int) -> None:
        self.set_i64(row, OFF_STEP, step)

    def step(self, row: int) -> int:
        return self.i64(row, OFF_STEP)

    def mark_lost(self, row: int) -> None:
        self.set_u32(row, OFF_LOST, 1)

    def lost(self, row: int) -> bool:
        return self.u32(row, OFF_LOST) != 0

    def set_order(self, row: int, members: list[int]) -> None:
        if len(members) > MAX_ROWS or len(set(members)) != len(members):
            raise ValueError(f"bad member order {members}")
        for m in members:
            if not 0 <= m < MAX_ROWS:
                raise ValueError(f"row {m} out of range")
        words = [len(members)] + list(members) + [0] * (MAX_ROWS - len(members))
        struct.pack_into("<9i", self.mm, self._off(row, OFF_ORDER), *words)

    def order(self, row: int) -> list[int]:
        words = struct.unpack_from("<9i", self.mm, self._off(row, OFF_ORDER))
        return list(words[1 : 1 + words[0]])

    def publish(self, row: int, handle: bytes) -> None:
        if len(handle) != HANDLE_BYTES:
            raise ValueError("IPC handles are 64 bytes")
        off = self._off(row, OFF_HANDLE)
        self.mm[off : off + HANDLE_BYTES] = handle
        self.set_u32(row, OFF_PUBLISHED, 1)

    def handle(self, row: int, timeout_s: float = 60.0) -> bytes:
        t0 = time.monotonic()
        while not self.u32(row, OFF_PUBLISHED):
            if time.monotonic() - t0 > timeout_s:
                raise TimeoutError(f"row {row} never published its buffer")
            time.sleep(0.001)
        off = self._off(row, OFF_HANDLE)
        return bytes(self.mm[off : off + HANDLE_BYTES])

    def unpublish(self, row: int) -> None:
        self.set_u32(row, OFF_PUBLISHED, 0)

    # ---- device mapping ------------------------------------------------------------------------
    def map_device(self, ext) -> int:
        """Pin and map the region into the current device's address space; returns its base."""
        if not self._registered:
            import ctypes

            addr = ctypes.addressof(ctypes.c_char.from_buffer(self.mm))
            self._host_base = addr
            self._dev_base = ext.host_register_mapped(addr, SIZE)
            self._registered = True
        return self._dev_base

    def ctrl_device(self, row: int) -> int:
        if not self._registered:
            raise RuntimeError("map_device first")
        return self._dev_base + ROW0 + row * ROW_BYTES

    def close(self, ext=None, unlink: bool = False) -> None:
        if self._registered and ext is not None:
            try:
                ext.host_unregister(self._host_base)
            except Exception:  # noqa: BLE001 - best effort at shutdown
                pass
            self._registered = False
        try:
            self.mm.close()
        except BufferError:
            pass
        if unlink:
            try:
                os.unlink(self.path)
            except FileNotFoundError:
                pass
