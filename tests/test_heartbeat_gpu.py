"""Failure detection inside the collective kernels, on one GPU, with no fault injected on the device.

A two-member all-reduce is launched with both members' buffers in this process: member 1 never
enters the call (its words never arrive) and never beats. The waiting kernel must leave on its own:
within milliseconds with the dead status when a beat limit is set (member 1's heartbeat stands
still), or on the host's abort word when it is not. Both are bounded waits that return a status;
nothing traps and the context stays usable.
"""

import os
import threading
import time

import pytest
import torch

from everserve_b200 import _ext
from everserve_b200.parallel.slot import MAX_ROWS, OFF_BEAT, SlotRegion

pytestmark = pytest.mark.gpu

DEAD, ABORTED = 4, 2


@pytest.fixture
def pair():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    C = _ext.load()
    dev = torch.device("cuda:0")
    # the region must live in shared memory (the device maps its pages)
    region = SlotRegion.create(f"es_hb_test_{os.getpid()}")
    region.map_device(C)
    nbytes = int(C.comm_buffer_bytes())
    bufs = [torch.zeros(nbytes, dtype=torch.uint8, device=dev) for _ in range(2)]
    peers = torch.tensor([b.data_ptr() for b in bufs] + [0] * (MAX_ROWS - 2), dtype=torch.int64, device=dev)
    order = torch.tensor([2, 0, 1] + [0] * (MAX_ROWS - 2), dtype=torch.int32, device=dev)
    call = torch.zeros(2, dtype=torch.int32, device=dev)
    seqs = torch.zeros(8192, dtype=torch.int32, device=dev)
    beat = C.heartbeat_start(region.beat_address(0), 500)  # member 0 (this process) beats
    yield C, region, (peers, order, call, region.ctrl_device(0), 0, 0, seqs)
    C.heartbeat_stop(beat)
    torch.cuda.synchronize()
    region.close(C, unlink=True)


def _call(C, comm, n=4096):
    x = torch.ones(n, dtype=torch.bfloat16, device="cuda")
    out = torch.empty_like(x)
    t0 = time.monotonic()
    C.fdar(x, out, *comm)
    torch.cuda.synchronize()
    return time.monotonic() - t0, out


def test_a_silent_member_is_named_dead_by_the_kernel(pair):
    C, region, comm = pair
    beat0 = region.beat(0)
    time.sleep(0.01)
    assert region.beat(0) > beat0  # the native heartbeat thread runs
    assert region.beat(1) == 0
    region.set_beat_limit_us([0], 5000)
    for n in (4096, 3 << 18):  # the LL path and the flag path
        region.set_u32(0, 16, 0)  # status
        region.clear_late(0)
        dt, _ = _call(C, comm, n)
        assert region.status(0) == DEAD, (n, region.status(0))
        assert region.late(0) & 0b10
        assert dt < 1.0, dt  # milliseconds of beat limit, not the 5 s hard limit


def test_without_beats_the_abort_word_releases_the_wait(pair):
    C, region, comm = pair
    region.set_beat_limit_us([0], 0)
    region.set_u32(0, 16, 0)

    def abort():
        time.sleep(0.2)
        region.set_abort([0], 1)

    t = threading.Thread(target=abort)
    t.start()
    dt, _ = _call(C, comm)
    t.join()
    assert region.status(0) == ABORTED and 0.15 < dt < 3.0, (region.status(0), dt)
    region.set_abort([0], 0)
