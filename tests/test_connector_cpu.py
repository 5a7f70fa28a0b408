"""The engine's KV connector over a committed-KV object (`state/connector.py`), against a recording
fake: what each step commits (slots, counts, step), the fence `depth` steps back, the per-step
commits of a multi-step window, drain and finished."""

from everserve_b200.engine.scheduler import ScheduledReq, StepPlan
from everserve_b200.state.connector import StoreConnector


class FakeCKV:
    def __init__(self):
        self.commits, self.fences, self.done = [], [], []

    def commit(self, epoch, step, counts, slots):
        self.commits.append((epoch, step, dict(counts), list(slots)))

    def fence(self, step, timeout_s=30.0):
        self.fences.append(step)

    def finished(self, req_id):
        self.done.append(req_id)

    def close(self):
        self.done.append("<closed>")


def _plan(step, reqs):
    return StepPlan(step=step, is_prefill=False, reqs=reqs)


def test_each_step_commits_its_slots_and_fences_depth_back():
    ckv = FakeCKV()
    con = StoreConnector(ckv, block_size=4, epoch=3, depth=2)
    a = ScheduledReq("a", [5], 6, [10, 11], sample=True)      # position 6: block 11, offset 2
    b = ScheduledReq("b", [7, 8], 2, [20], sample=True)       # positions 2, 3 of block 20
    con.end_step(_plan(0, [a, b]), None)
    assert ckv.commits == [(3, 0, {"a": 7, "b": 4}, [46, 82, 83])]
    assert ckv.fences == []
    for step in (1, 2, 3):
        a = ScheduledReq("a", [1], 6 + step, [10, 11, 12], sample=True)
        con.end_step(_plan(step, [a]), None)
    # a commit is fenced once `depth` newer ones are in flight
    assert ckv.fences == [0, 1]
    assert [c[1] for c in ckv.commits] == [0, 1, 2, 3]
    assert con.commits == 4
    con.drain()
    assert ckv.fences[-1] == 3


def test_decode_window_commits_every_device_step():
    ckv = FakeCKV()
    con = StoreConnector(ckv, block_size=4, epoch=1, depth=2)
    reqs = [ScheduledReq("a", [1], 3, [5, 6], sample=True), ScheduledReq("b", [2], 8, [7, 8, 9], sample=True)]
    hook = con.decode_hook(_plan(40, reqs), 3)
    for i in range(3):
        hook(i)
    assert [c[1] for c in ckv.commits] == [40, 41, 42]
    # step i writes position start + i of every request
    assert ckv.commits[0][3] == [5 * 4 + 3, 9 * 4 + 0]
    assert ckv.commits[1][3] == [6 * 4 + 0, 9 * 4 + 1]
    assert ckv.commits[2][3] == [6 * 4 + 1, 9 * 4 + 2]
    assert ckv.commits[2][2] == {"a": 6, "b": 11}
    assert ckv.fences == [40]


def test_finished_and_close():
    ckv = FakeCKV()
    con = StoreConnector(ckv, block_size=16)
    con.finished("x")
    con.end_step(_plan(5, [ScheduledReq("y", [1], 0, [3], sample=True)]), None)
    con.close()
    assert ckv.done == ["x", "<closed>"]
    assert ckv.fences == [5]  # close drains first
