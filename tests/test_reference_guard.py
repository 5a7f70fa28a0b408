"""The reference tier's step guard on gloo ranks: a rank dies in the middle of a step.

Four ranks run the placement-independent decoder under ``StepGuard``. At decode step 3 rank 2
exits after its first collective of the step (host-side: the process ends itself; nothing of it
is on a device). The survivors' collective fails, they abandon the attempt and roll back what it
wrote; the parent sees rank 2 go and sends the fault; the survivors form their group, absorb rank
2's units with its KV up to the last accepted step, and run step 3 again. Every step's logits
equal the single-process oracle's bit for bit.

A second test has one member accept a step the others did not, and checks that it replays the
step for them after a recovery.
"""

import datetime
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from everserve_b200.reference import plan as P
from everserve_b200.reference.control import FaultListener, broadcast_fault
from everserve_b200.reference.cores import LlamaCore
from everserve_b200.reference.guard import StepGuard
from everserve_b200.reference.store import ExactStore, LoopbackCommittedKV

from test_reference_tier import CFG, MLP_UNITS, MOE, WORLD, _oracle, _steps

DIE_STEP, DIE_AT_CALL = 3, 2


def _guarded_rank(rank, cfg, port, store_addr, conn, fault_q, die):
    torch.set_num_threads(1)
    tcp = dist.TCPStore("127.0.0.1", port, is_master=False, timeout=datetime.timedelta(seconds=60))
    from everserve_b200.reference.world import form_group, shrink_world

    group = form_group(tcp, list(range(WORLD)), rank, timeout_s=20)
    place = {"attn": P.even_units(cfg.kv_heads, WORLD), "mlp": P.even_units(MLP_UNITS, WORLD)}
    kv = LoopbackCommittedKV(store_addr)
    faults = FaultListener()
    fault_q.put((rank, faults.address))
    now = {"step": -1, "calls": 0}
    written = {}

    def reduce(t):
        now["calls"] += 1
        if die and rank == 2 and now["step"] == DIE_STEP and now["calls"] == DIE_AT_CALL:
            os._exit(3)  # dies in the middle of the step, after its first collective
        return guard.all_reduce(t)

    core = LlamaCore(cfg, rank, place["attn"][rank], place["mlp"][rank], MLP_UNITS, reduce=reduce)

    def leave(f):
        shrink_world(group, f["lost"], f["epoch"])

    def absorb(f, upto):
        a1, m1 = P.after_loss(place["attn"], f["lost"]), P.after_loss(place["mlp"], f["lost"])
        ga, gm = P.moved(place["attn"], a1)[rank], P.moved(place["mlp"], m1)[rank]
        core.absorb(ga, gm, kv.restore(ga, upto))
        place["attn"], place["mlp"] = a1, m1

    guard = StepGuard(group, leave, absorb, faults, confirm_timeout_s=30)
    marks = {}
    guard.attempt_callbacks.append(lambda: marks.__setitem__("attempt", core.mark()))
    guard.abandon_callbacks.append(lambda: core.rollback(marks["attempt"]))
    guard.accept_callbacks.append(lambda: marks.__setitem__("last", marks["attempt"]))
    guard.replay_callbacks.append(lambda: core.rollback(marks["last"]))
    guard.commit_callbacks.append(lambda: kv.commit(rank, guard.epoch, written["step"], written["rows"]))

    def step_fn(k, s):
        def fn():
            now["calls"] = 0
            logits, rows = core.forward(*s)
            written["step"], written["rows"] = k, rows
            return logits
        return fn

    for k, s in enumerate(_steps()):
        conn.recv()
        now["step"] = k
        conn.send(guard.run_step(step_fn(k, s)))
    conn.send([e[1] for e in guard.events])
    conn.recv()  # the parent has read every tensor (they are shared through this process)


@pytest.mark.parametrize("cfg", [CFG, MOE], ids=["dense", "moe"])
def test_rank_dies_mid_step_survivors_rerun_bit_identical(cfg):
    expect = _oracle(cfg)
    ctx = mp.get_context("spawn")
    tcp = dist.TCPStore("127.0.0.1", 0, is_master=True, wait_for_workers=False)
    store = ExactStore()
    q = ctx.Queue()
    pipes, procs = [], []
    for r in range(WORLD):
        a, b = ctx.Pipe()
        p = ctx.Process(target=_guarded_rank, args=(r, cfg, tcp.port, store.address, b, q, True))
        p.start()
        pipes.append(a)
        procs.append(p)
    faults = dict(q.get(timeout=60) for _ in range(WORLD))
    alive = list(range(WORLD))
    try:
        for step in range(len(_steps())):
            for r in alive:
                pipes[r].send("step")
            if step == DIE_STEP:
                procs[2].join(timeout=60)
                assert procs[2].exitcode == 3
                alive.remove(2)
                broadcast_fault([faults[r] for r in alive], {"lost": [2], "epoch": 1})
            for r in alive:
                assert pipes[r].poll(120), f"rank {r} did not finish step {step}"
                assert torch.equal(pipes[r].recv(), expect[step]), f"rank {r} step {step} differs"
        events = [pipes[r].recv() for r in alive]
        for r in alive:
            pipes[r].send("bye")
        for ev in events:
            assert "failed" in ev or "aborted" in ev  # the attempt of step 3 was abandoned
            assert ev.count("recover") == 1 and "replayed" not in ev
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
        store.close()


def _reconcile_rank(rank, port, conn):
    torch.set_num_threads(1)
    tcp = dist.TCPStore("127.0.0.1", port, is_master=False, timeout=datetime.timedelta(seconds=60))
    from everserve_b200.reference.world import form_group

    group = form_group(tcp, [0, 1, 2], rank, timeout_s=20)
    state = {"x": torch.zeros(4)}
    marks = {}
    guard = StepGuard(group, leave=lambda f: None, absorb=lambda f, upto: None)
    guard.attempt_callbacks.append(lambda: marks.__setitem__("attempt", state["x"].clone()))
    guard.abandon_callbacks.append(lambda: state.__setitem__("x", marks["attempt"]))
    guard.accept_callbacks.append(lambda: marks.__setitem__("last", marks["attempt"]))
    guard.replay_callbacks.append(lambda: state.__setitem__("x", marks["last"]))

    def step(k):
        def fn():
            t = torch.full((4,), float(k + 1) * (rank + 1))
            guard.all_reduce(t)
            state["x"] = state["x"] + t
            return state["x"].clone()
        return fn

    outs = [guard.run_step(step(0)), guard.run_step(step(1))]
    if rank == 0:
        # as if the agreement of step 2 completed on rank 0 only: it accepted step 2, the others
        # abandoned it (their state is the one before it)
        marks["last"] = state["x"].clone()
        state["x"] = state["x"] + torch.full((4,), 3.0 * 6)
        guard.accepted += 1
        guard._last_fn = step(2)
        outs.append(state["x"].clone())
    guard.flag({"lost": [], "epoch": 1})
    if rank != 0:
        outs.append(guard.run_step(step(2)))  # re-run: rank 0 replays it with them
    outs.append(guard.run_step(step(3)))
    conn.send((outs, [e[1] for e in guard.events]))
    conn.recv()


def test_member_ahead_replays_the_step_the_others_rerun():
    ctx = mp.get_context("spawn")
    tcp = dist.TCPStore("127.0.0.1", 0, is_master=True, wait_for_workers=False)
    pipes, procs = [], []
    for r in range(3):
        a, b = ctx.Pipe()
        p = ctx.Process(target=_reconcile_rank, args=(r, tcp.port, b))
        p.start()
        pipes.append(a)
        procs.append(p)
    try:
        got = []
        for a in pipes:
            assert a.poll(120)
            got.append(a.recv())
        for a in pipes:
            a.send("bye")
        outs = [g[0] for g in got]
        # every step k adds (k + 1) * (1 + 2 + 3) to each element
        want = [torch.full((4,), 6.0 * sum(range(1, k + 2))) for k in range(4)]
        for o in outs:
            assert all(torch.equal(a, b) for a, b in zip(o, want))
        assert "replayed" in got[0][1] and "replayed" not in got[1][1]
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
