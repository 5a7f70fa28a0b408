"""Host-side runtime pieces: the failure detector, layouts, policy, discovery and the daemon contract."""

import os
import subprocess
import sys
import time

import pytest

from everserve_b200 import discovery, policy
from everserve_b200.outcome import Outcome
from everserve_b200.parallel.slot import SlotRegion
from everserve_b200.runtime.layout import ParallelLayout, Scope, position, replacement
from everserve_b200.runtime.slotwatch import SlotWatch, process_state


@pytest.fixture
def region(tmp_path):
    r = SlotRegion(str(tmp_path / "slot"), create=True)
    yield r
    r.close()


def _sleeper():
    return subprocess.Popen([sys.executable, "-c", "import time; time.sleep(60)"])


def test_process_state_dead_alive_zombie():
    p = _sleeper()
    try:
        assert process_state(p.pid) == "alive"
        p.kill()
        time.sleep(0.05)
        assert process_state(p.pid) == "dead"  # a zombie until reaped
    finally:
        p.wait()
    assert process_state(p.pid) == "dead"
    assert process_state(os.getpid()) == "alive"


def test_slotwatch_reports_dead_member_within_ms(region):
    p = _sleeper()
    lost = []
    try:
        region.set_pid(0, os.getpid())
        region.set_pid(1, p.pid)
        w = SlotWatch(region, 0, lambda ranks, why: lost.append((time.monotonic(), ranks, why)), members=[0, 1],
                      hang_s=60).start()
        region.set_u32(0, 4, 0b10)  # the kernel named row 1 late
        time.sleep(0.05)
        assert lost == []  # late but alive: not yet hung
        t_kill = time.monotonic()
        p.kill()
        deadline = time.monotonic() + 2
        while not lost and time.monotonic() < deadline:
            time.sleep(0.001)
        w.stop()
    finally:
        p.wait()
    assert lost and lost[0][1] == [1] and lost[0][2] == "dead"
    assert (lost[0][0] - t_kill) < 0.5
    assert region.lost(1)


def test_slotwatch_hung_after_hang_s(region):
    p = _sleeper()
    lost = []
    try:
        region.set_pid(1, p.pid)
        w = SlotWatch(region, 0, lambda ranks, why: lost.append((ranks, why)), members=[0, 1], hang_s=0.1)
        region.set_u32(0, 4, 0b10)
        t0 = time.monotonic()
        while not lost and time.monotonic() - t0 < 2:
            w.check()
            time.sleep(0.005)
        assert lost == [([1], "hung")]
    finally:
        p.kill()
        p.wait()


def test_slotwatch_step_stall_finds_dead_member(region):
    p = _sleeper()
    lost = []
    region.set_pid(0, os.getpid())
    region.set_pid(1, p.pid)
    p.kill()
    p.wait()
    w = SlotWatch(region, 0, lambda ranks, why: lost.append((ranks, why)), members=[0, 1], stall_s=0.05)
    region.set_step(0, 7)
    t0 = time.monotonic()
    while not lost and time.monotonic() - t0 < 2:
        w.check()
        time.sleep(0.005)
    assert lost and lost[0][0] == [1]


def test_layout_positions_and_members():
    lay = ParallelLayout(tensor_parallel=2, pipeline_parallel=2)
    assert lay.world == 4
    assert [lay.stage(r) for r in range(4)] == [0, 0, 1, 1]
    assert [lay.column(r) for r in range(4)] == [0, 1, 0, 1]
    members = [0, 1, replacement(2), 3]
    assert lay.tensor_members(members, 3) == ("R2", 3)
    assert lay.pipeline_members(members, 0) == (0, "R2")
    assert lay.members_of(Scope.DOMAIN, members, 0) == (0, 1)
    assert position("R2") == 2
    assert lay.next_stage(1) == 3 and lay.prev_stage(3) == 1 and lay.next_stage(3) is None
    assert lay.last_stage_ranks() == [2, 3]


def test_policy_outcomes_and_sets():
    p = policy.from_json('{"outcomesInOrder": ["OUTCOME_REPLACE", "OUTCOME_SHRINK"], "engines": ['
                         '{"name": "e0", "tensorParallel": 4, "placementIndependentModel": true,'
                         ' "spares": [{"node": "n1", "device": 4, "rank": 2}]}]}')
    e = p.engine("e0")
    assert e.world_size == 4 and e.spare_ranks == (2,) and e.spare_node(2) == "n1"
    assert policy.choose_outcome(p, spare_ready=True, placement_independent_model=False) is Outcome.REPLACE
    assert policy.choose_outcome(p, spare_ready=False, placement_independent_model=True) is Outcome.SHRINK
    assert policy.choose_outcome(p, spare_ready=False, placement_independent_model=False) is Outcome.REBUILD
    sets = policy.sets_to_preform(p, e, e.spare_ranks)
    assert sets[:4] == [(1, 2, 3), (0, 2, 3), (0, 1, 3), (0, 1, 2)]
    assert sets[4] == (0, 1, "R2", 3)
    with pytest.raises(ValueError):
        policy.sets_to_preform(p, e, [9])
    with pytest.raises(KeyError):
        p.engine("nope")


def test_discovery_file_backend(tmp_path, monkeypatch):
    d = discovery.FileDiscovery(tmp_path)
    d.publish(discovery.DaemonRecord("n0", "unix:/run/n0.sock", ("e0",), 5, 42, "unix:/run/s.sock", "10.0.0.1"))
    rec = d.daemon("n0")
    assert rec.address == "unix:/run/n0.sock" and rec.mirror_address == "unix:/run/s.sock" and rec.host == "10.0.0.1"
    monkeypatch.delenv(discovery.DAEMON_SOCKET_ENV, raising=False)
    assert discovery.local_daemon("n0", tmp_path).pid == 42
    monkeypatch.setenv(discovery.DAEMON_SOCKET_ENV, "unix:/x.sock")
    assert discovery.local_daemon("n0").address == "unix:/x.sock"


def test_a_release_past_its_bound_is_reported_as_a_leak():
    import threading
    import time

    import torch

    from everserve_b200.runtime.groups import SwappableGroups
    from everserve_b200.runtime.layout import ParallelLayout

    class Stuck:
        epoch = 3

        def __init__(self, seconds):
            self.seconds = seconds

        def abort(self):
            time.sleep(self.seconds)

    leaks = []
    got = threading.Event()
    g = SwappableGroups(None, 0, ParallelLayout(1, 1), torch.device("cpu"), release_bound_s=0.2,
                        on_leak=lambda what, s, n: (leaks.append((what, s, n)), got.set()))
    g._release(Stuck(0.0), "fast")
    g._release(Stuck(2.0), "epoch 3 groups")
    assert got.wait(5)
    assert leaks[0][0] == "epoch 3 groups" and leaks[0][1] >= 0.2 and leaks[0][2] == 1
    time.sleep(0.3)
    assert len(leaks) == 1  # the fast release was no leak


def test_slotwatch_names_a_member_whose_heartbeat_stopped(tmp_path, monkeypatch):
    """A member's beat word that stands still past the limit is a death, even when no kernel has
    named it late (its process may look alive to /proc for a moment: a zombie, a frozen host)."""
    import os
    import time

    from everserve_b200.parallel.slot import OFF_BEAT, SlotRegion
    from everserve_b200.runtime import slotwatch as sw

    monkeypatch.setenv("EVERSERVE_SHM_DIR", str(tmp_path))
    region = SlotRegion.create("beats")
    for row in (0, 1, 2):
        region.set_pid(row, os.getpid())  # every member "alive" to the /proc check
    lost = []
    w = sw.SlotWatch(region, 0, lambda ranks, why: lost.append((ranks, why)), members=[0, 1, 2],
                     beat_limit_s=0.05)
    t0 = time.monotonic()
    while time.monotonic() - t0 < 1.0 and not lost:
        region.set_u32(2, OFF_BEAT, region.beat(2) + 1)  # row 2 beats, row 1 does not
        w.check()
        time.sleep(0.005)
    assert lost == [([1], "dead")]
    assert time.monotonic() - t0 < 0.5
    region.close(unlink=True)
