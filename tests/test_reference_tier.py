"""The CPU reference tier: placement plans, and SHRINK with bit-identical outputs.

Four gloo ranks serve a decoder whose work is split into units (one KV head each, MLP slices).
Between two decode steps rank 2 leaves (its process exits; nothing of it in flight). The parent,
acting as the head, sees it go and sends the survivors a fault over the fault channel; they form
the survivors' group, absorb rank 2's units by the after-loss plan (weights from the deterministic
source, KV rows of its heads from the exact store) and continue. Every step's logits equal the
single-process oracle's bit for bit.
"""

import datetime
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from everserve_b200.models.config import ModelConfig
from everserve_b200.reference import plan as P
from everserve_b200.reference.control import FaultListener, broadcast_fault
from everserve_b200.reference.cores import LlamaCore
from everserve_b200.reference.recapture import next_slice
from everserve_b200.reference.staging import blocks_to_stage
from everserve_b200.reference.store import ExactStore, LoopbackCommittedKV

CFG = ModelConfig(name="ref-tiny", vocab=64, hidden=32, layers=2, heads=8, kv_heads=4, head_dim=8, intermediate=64,
                  rope_theta=1e4, rms_eps=1e-6)
MOE = ModelConfig(name="ref-moe", vocab=64, hidden=32, layers=2, heads=8, kv_heads=4, head_dim=8, intermediate=16,
                  rope_theta=1e4, rms_eps=1e-6, num_experts=8, top_k=2)
WORLD, MLP_UNITS = 4, 8


def _steps():
    """A prefill of two sequences, then decode steps (tokens fixed, not sampled)."""
    g = torch.Generator().manual_seed(3)
    prefill = (torch.randint(0, 64, (8,), generator=g), torch.tensor([0, 1, 2, 3, 4, 0, 1, 2]),
               torch.tensor([0, 0, 0, 0, 0, 1, 1, 1]))
    out = [prefill]
    for k in range(5):
        out.append((torch.randint(0, 64, (2,), generator=g), torch.tensor([5 + k, 3 + k]), torch.tensor([0, 1])))
    return out


def test_plans():
    assert P.even_units(8, 4) == {0: [0, 1], 1: [2, 3], 2: [4, 5], 3: [6, 7]}
    with pytest.raises(ValueError):
        P.even_units(7, 4)
    assert P.expert_chunks(8, 2, 2) == {0: [(0, 1), (2, 3)], 1: [(4, 5), (6, 7)]}
    after = P.after_loss(P.even_units(8, 4), [2])
    assert sorted(u for us in after.values() for u in us) == list(range(8))
    assert after == {0: [0, 1, 4], 1: [2, 3, 5], 3: [6, 7]}
    assert P.moved(P.even_units(8, 4), after) == {0: [4], 1: [5], 3: []}
    assert P.capacity_after_one_loss(8, 4, 3) and not P.capacity_after_one_loss(8, 4, 2)
    assert blocks_to_stage([(7, 3), (2, 1), (5, 2)], 2) == [[2, 5], [7]]
    assert next_slice([1, 2, 4, 8, 16], {4}, 4) == 8
    assert next_slice([1, 2, 4], {1, 2, 4}, 2) is None


def _oracle(cfg):
    torch.set_num_threads(1)
    core = LlamaCore(cfg, 0, range(cfg.kv_heads), range(MLP_UNITS), MLP_UNITS)
    return [core.forward(*s)[0] for s in _steps()]


def _rank(rank, cfg, port, store_addr, conn, fault_addr_q):
    torch.set_num_threads(1)
    tcp = dist.TCPStore("127.0.0.1", port, is_master=False, timeout=datetime.timedelta(seconds=30))
    from everserve_b200.reference.world import form_group, shrink_world

    group = form_group(tcp, list(range(WORLD)), rank)
    attn0, mlp0 = P.even_units(cfg.kv_heads, WORLD), P.even_units(MLP_UNITS, WORLD)
    core = LlamaCore(cfg, rank, attn0[rank], mlp0[rank], MLP_UNITS, reduce=group.all_reduce)
    kv = LoopbackCommittedKV(store_addr)
    faults = FaultListener()
    fault_addr_q.put((rank, faults.address))
    epoch = 0
    for step, s in enumerate(_steps()):
        cmd = conn.recv()
        if cmd == "exit":
            os._exit(0)  # leaves between steps
        if cmd == "check-fault":
            f = faults.next(timeout=30)
            lost, epoch = f["lost"], f["epoch"]
            shrink_world(group, lost, epoch)
            a1, m1 = P.after_loss(attn0, lost), P.after_loss(mlp0, lost)
            gained_a, gained_m = P.moved(attn0, a1)[rank], P.moved(mlp0, m1)[rank]
            core.absorb(gained_a, gained_m, kv.restore(gained_a))
            conn.recv()  # the step command
        logits, rows = core.forward(*s)
        kv.commit(rank, epoch, step, rows)
        conn.send(logits)
    conn.close()


@pytest.mark.parametrize("cfg", [CFG, MOE], ids=["dense", "moe"])
def test_shrink_bit_identical(cfg):
    expect = _oracle(cfg)
    ctx = mp.get_context("spawn")
    tcp = dist.TCPStore("127.0.0.1", 0, is_master=True, wait_for_workers=False)
    store = ExactStore()
    q = ctx.Queue()
    pipes, procs = [], []
    for r in range(WORLD):
        a, b = ctx.Pipe()
        p = ctx.Process(target=_rank, args=(r, cfg, tcp.port, store.address, b, q))
        p.start()
        pipes.append(a)
        procs.append(p)
    faults = dict(q.get(timeout=60) for _ in range(WORLD))
    alive = list(range(WORLD))
    try:
        for step in range(len(_steps())):
            if step == 3:  # rank 2 leaves between steps 2 and 3
                pipes[2].send("exit")
                procs[2].join(timeout=30)
                assert procs[2].exitcode == 0
                alive.remove(2)
                for r in alive:
                    pipes[r].send("check-fault")
                broadcast_fault([faults[r] for r in alive], {"lost": [2], "epoch": 1})
            for r in alive:
                pipes[r].send("step")
            outs = [pipes[r].recv() for r in alive]
            for o in outs:
                assert torch.equal(o, expect[step]), f"step {step} differs"
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
        store.close()
