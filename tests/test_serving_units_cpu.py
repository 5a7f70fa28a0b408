"""Unit checks of three serving-path rules, with fakes (no processes, no GPU):

* which staging directories the KV commit pins in place (tmpfs only);
* a serving rank's collective wait bound: the hung-member limit until the step period is
  measured, then `detect_steps` median periods with the floor, re-measured every `step_sample`
  steps and back to the limit at a membership change;
* the head's handling of a step a rank answered with an error: it reports the loss to the
  coordinator (unless a change for a fault is under way) and, when no change follows, ends in
  EngineDown naming the rank's error.
"""

import threading

import pytest

from everserve_b200.serving.executor import EngineDown, MultiprocExecutor, RankLost
from everserve_b200.serving.rank import RankProcess
from everserve_b200.settings import Settings
from everserve_b200.state.mirror import pinnable

MOUNTS = """overlay / overlay rw,relatime 0 0
tmpfs /dev/shm tmpfs rw,nosuid,nodev 0 0
/dev/vda1 /data ext4 rw,relatime 0 0
tmpfs /data/fast tmpfs rw 0 0
/dev/vdb /mnt/with\\040space xfs rw 0 0
"""


def test_pinnable_only_on_tmpfs():
    assert pinnable("/dev/shm/everserve/eng/rank0", MOUNTS)
    assert pinnable("/data/fast/store", MOUNTS)  # the longest mount point wins
    assert not pinnable("/data/store", MOUNTS)
    assert not pinnable("/tmp/pytest-of-root/x", MOUNTS)  # the overlay root
    assert not pinnable("/dev/shmother", MOUNTS)  # a prefix of a name is not its mount
    assert not pinnable("/mnt/with space/d", MOUNTS)


class FakeCollective:
    def __init__(self):
        self.bounds = []

    def set_bound_ns(self, ns):
        self.bounds.append(ns)


def test_rank_bound_follows_the_measured_step_period():
    s = Settings(detect_steps=3.0, detect_floor_ms=30.0, hang_s=10.0, step_sample=4)
    assert s.warmup_bound_ns() == 10_000_000_000
    r = RankProcess.__new__(RankProcess)  # only the sampling rule: no process, no device
    r.settings, r.collective, r._step_dt = s, FakeCollective(), []
    for dt in (0.5, 0.020, 0.021, 0.019):  # a slow first step, then 20 ms steps
        r._sample_step(dt)
    assert r.collective.bounds == [int(3 * 0.021 * 1e9)]  # three median periods: 63 ms
    for dt in (0.004, 0.005, 0.004, 0.006):  # faster steps: the floor holds
        r._sample_step(dt)
    assert r.collective.bounds[-1] == 30_000_000
    assert r._step_dt == []


class FakeClient:
    def __init__(self, commit=False):
        self.reports = []
        self.commit = commit
        self.pending_change = threading.Event()
        self.last_change = None

    def report_lost(self, ranks, detail="", epoch=0):
        self.reports.append((list(ranks), detail))

    def wait_committed(self, timeout_s=None, after_epoch=0):
        raise TimeoutError(f"no membership commit within {timeout_s} s")


def _head(client):
    ex = MultiprocExecutor.__new__(MultiprocExecutor)  # only the change rule
    ex.client, ex.change_timeout_s, ex.epoch = client, 0.1, 0
    return ex


def test_head_reports_a_failed_step_and_names_it():
    client = FakeClient()
    ex = _head(client)
    cause = RankLost([1], "rank 1: RuntimeError: a collective of step 3 failed (status 1)")
    with pytest.raises(EngineDown, match="status 1"):
        ex.complete_change(None, cause=cause)
    assert client.reports == [([1], "step failed on the rank: rank 1: RuntimeError: a collective of step 3 "
                                    "failed (status 1)")]


def test_head_does_not_report_when_a_fault_change_is_under_way():
    client = FakeClient()

    class Change:
        epoch, lost, departing = 1, [1], []

    client.last_change = Change()
    client.pending_change.set()
    ex = _head(client)
    with pytest.raises(EngineDown):
        ex.complete_change(None, cause=RankLost([1], "link ended"))
    assert client.reports == []
