"""Descriptor exchange of the symmetric peer buffers, on the CPU with a stand-in for the driver calls.

A member that maps a peer's buffer may ask before the peer has created it (the peer is still
loading its weights, say). The mapping must wait for the peer's socket instead of failing, and
still give up with an error once its timeout has passed.
"""

import os
import threading
import time

import pytest

from everserve_b200.parallel.symm import PeerMapping, SymmetricBuffer


class FakeDriver:
    """vmm_create hands out a real descriptor (of /dev/null) so SCM_RIGHTS has something to pass."""

    def __init__(self):
        self.imported = []
        self.released = []

    def vmm_create(self, nbytes):
        return (0x1000, nbytes, 7, os.open("/dev/null", os.O_RDONLY))

    def vmm_import(self, fd, size):
        self.imported.append(size)
        return (0x2000, size, 9)

    def vmm_release(self, ptr, size, handle, fd):
        self.released.append((ptr, handle))
        if fd >= 0:
            os.close(fd)


def test_mapping_waits_for_a_late_peer(tmp_path):
    C = FakeDriver()
    path = str(tmp_path / "region.r1.moe0.fd")
    made = {}

    def late_peer():
        time.sleep(0.3)
        made["buf"] = SymmetricBuffer(C, 4096, path)

    t = threading.Thread(target=late_peer)
    t.start()
    m = PeerMapping(C, path, timeout_s=10.0)
    t.join()
    assert (m.ptr, m.size) == (0x2000, 4096)
    assert C.imported == [4096]
    m.close()
    made["buf"].close()
    assert (0x2000, 9) in C.released and (0x1000, 7) in C.released


def test_mapping_gives_up_after_its_timeout(tmp_path):
    C = FakeDriver()
    t0 = time.monotonic()
    with pytest.raises((FileNotFoundError, ConnectionRefusedError)):
        PeerMapping(C, str(tmp_path / "never.fd"), timeout_s=0.2)
    assert time.monotonic() - t0 < 5.0
