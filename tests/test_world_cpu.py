"""World re-form and group shrink on the CPU (gloo ranks).

* constant world size: both ranks leave their default group and join a fresh rendezvous, where a
  collective works again;
* SHRINK by NCCL shrink: a stand-in for ``torch.distributed.shrink_group`` records the call (the
  lost ranks by group rank, with the abort flag); when it fails the group is re-formed over the store
  and the failure kept.
"""

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from everserve_b200.reference.world import join_world, leave_world
from everserve_b200.runtime import shrink as shrink_mod


def _port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _reform(rank: int, p1: int, p2: int, out):
    join_world(f"tcp://127.0.0.1:{p1}", rank, 2, "gloo", datetime.timedelta(seconds=30))
    t = torch.ones(1) * (rank + 1)
    dist.all_reduce(t)
    first = float(t)
    steps = leave_world()
    join_world(f"tcp://127.0.0.1:{p2}", rank, 2, "gloo", datetime.timedelta(seconds=30))
    t = torch.ones(1) * 10 * (rank + 1)
    dist.all_reduce(t)
    out[rank] = (first, steps, float(t))
    leave_world()


def test_leave_and_join_a_new_world():
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    p1, p2 = _port(), _port()
    ps = [ctx.Process(target=_reform, args=(r, p1, p2, out)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in ps), [p.exitcode for p in ps]
    for r in range(2):
        first, steps, second = out[r]
        assert first == 3.0 and second == 30.0 and steps == ["destroy"]


def test_leave_without_a_world_does_nothing():
    assert not dist.is_initialized()
    assert leave_world() == []


class _FakePG:
    def __init__(self):
        self.aborted = False

    def abort(self):
        self.aborted = True


def test_nccl_shrink_excludes_the_lost_by_group_rank(monkeypatch):
    calls = []
    new_pg = object()

    def fake_shrink(ranks_to_exclude, group=None, shrink_flags=0, pg_options=None):
        calls.append((list(ranks_to_exclude), group, shrink_flags))
        return new_pg

    monkeypatch.setattr(dist, "shrink_group", fake_shrink, raising=False)
    old = _FakePG()
    g = shrink_mod.ShrinkableGroup.from_group(old, members=[3, 5, 7, 9], me=5, backend="nccl")
    g.shrink([7, 9], epoch=4)
    from torch.distributed import distributed_c10d as c10d

    assert calls == [([2, 3], old, c10d.SHRINK_ABORT)]
    assert g.pg is new_pg and g.members == [3, 5] and g.rank == 1 and g.method == shrink_mod.NCCL_SHRINK
    assert g.epoch == 4 and g.shrink_failure is None


def test_failed_nccl_shrink_falls_back_to_recreate(monkeypatch):
    def failing(ranks_to_exclude, group=None, shrink_flags=0, pg_options=None):
        raise RuntimeError("ncclCommShrink unsupported")

    formed = []
    monkeypatch.setattr(dist, "shrink_group", failing, raising=False)
    monkeypatch.setattr(shrink_mod.ShrinkableGroup, "_form", lambda self: formed.append(list(self.members)) or "pg")
    old = _FakePG()
    g = shrink_mod.ShrinkableGroup.from_group(old, members=[0, 1, 2], me=0, backend="nccl", store=object())
    g.shrink([2], epoch=1)
    assert old.aborted and formed == [[0, 1]] and g.method == shrink_mod.RECREATE
    assert "ncclCommShrink unsupported" in g.shrink_failure


def test_shrink_refuses_strangers_and_self():
    g = shrink_mod.ShrinkableGroup.from_group(_FakePG(), members=[0, 1], me=0, backend="nccl")
    with pytest.raises(ValueError):
        g.shrink([5], epoch=1)
    with pytest.raises(ValueError):
        g.shrink([0], epoch=1)
