"""Failover on the CPU tier: a pipeline-parallel engine loses a rank mid-decode and a spare takes it.

TP1 PP2 (world size 2) plus one spare standing for rank 1, with the C++ coordinator, node daemon
and KV store. Rank 1 is SIGKILLed at decode step 20; the coordinator replaces it with the spare,
which restores rank 1's committed KV from the store; the engine resumes every stream from its
committed tokens and every stream must complete token-identical to the no-fault run.

The default runs a narrow model of the same architecture (fast); ``ES_FULL_CONFIG1=1`` runs the
full Qwen2.5-0.5B shape (24 layers, hidden 896, vocab 151936) with 8 streams x 128-token prompts
and 64 greedy tokens, the reference's own configuration.
"""

import os
import random

import pytest
import torch

from everserve_b200.engine.config import EngineConfig
from everserve_b200.engine.engine import Engine
from everserve_b200.models.config import get_config
from everserve_b200.serving.cluster import ControlPlane
from everserve_b200.serving.executor import MultiprocExecutor, failover

FULL = os.environ.get("ES_FULL_CONFIG1") == "1"
MODEL = "qwen2.5-0.5b" if FULL else "tiny-qwen"
STREAMS, PROMPT, TOKENS, KILL_AT = 8, 128, (64 if FULL else 28), 20


def _prompts():
    rng = random.Random(0)
    vocab = get_config(MODEL).vocab
    return [[rng.randrange(vocab) for _ in range(PROMPT)] for _ in range(STREAMS)]


def _run(workdir, kill_at=None, spares=(1,), kill_prefill=None, **sampling):
    cfg = EngineConfig(model=MODEL, device="cpu", dtype=torch.float32, num_blocks=128, max_batch=STREAMS,
                       max_model_len=PROMPT + TOKENS + 16, pipeline_parallel=2, use_cuda_graphs=False)
    with ControlPlane(str(workdir), engines=[{"name": "e0", "pipelineParallel": 2}]) as cp:
        ex = MultiprocExecutor(cfg, engine="e0", daemon=cp.daemon_socket, store=cp.store_socket, spares=spares,
                               node="n0", log_dir=str(workdir / "logs"), threads=2)
        try:
            if spares:
                cp.wait_spares("e0", len(spares))
                _wait_covered(cp, "e0")
            eng = Engine(cfg, executor=ex)
            eng.wrap_step(failover(ex, eng))
            if kill_at is not None:
                ex.kill_at_decode_step = kill_at if isinstance(kill_at, tuple) else (kill_at, 1)
            if kill_prefill is not None:
                ex.kill_at_prefill_step = kill_prefill
            out = eng.generate(_prompts(), max_tokens=TOKENS, **sampling)
            mism = sum(r.replay_mismatches for r in eng.scheduler.requests.values())
            view = cp.engine_view("e0")
            return out, ex.changes, mism, view
        finally:
            ex.shutdown()


def _wait_covered(cp, engine, timeout_s=60.0):
    """The coordinator's cover plan for the spare is formed by every member."""
    import time

    deadline = time.monotonic() + timeout_s
    while time.monotonic() < deadline:
        sets = cp.engine_view(engine)["status"]["cover"]["sets"]
        if any(s["covers"] and s["covered"] for s in sets):
            return
        time.sleep(0.05)
    raise TimeoutError(f"no covered replacement set: {cp.engine_view(engine)['status']['cover']}")


@pytest.mark.slow
def test_sigkill_rank1_spare_takes_over_token_identical(tmp_path):
    base, changes0, _, _ = _run(tmp_path / "nofault", spares=())
    assert changes0 == []
    events = tmp_path / "events"
    os.environ["EVERSERVE_EVENT_DIR"] = str(events)  # the rank processes write their event logs
    try:
        out, changes, mism, view = _run(tmp_path / "fault", kill_at=KILL_AT)
    finally:
        del os.environ["EVERSERVE_EVENT_DIR"]
    assert len(changes) == 1
    rec = changes[0].as_dict()
    sp = rec["spans"]
    assert all(sp[k] is not None and sp[k] >= 0 for k in ("decide", "acks", "commit", "claim_to_commit"))
    assert abs(sp["decide"] + sp["acks"] + sp["commit"] - sp["claim_to_commit"]) < 0.01
    assert len(rec["first_steps_ms"]) == 3
    import json

    trace = [json.loads(line) for line in open(events / "rank0.trace.jsonl")]
    kinds = [t["kind"] for t in trace]
    assert "change" in kinds and "boundary" in kinds and all("wall" in t and "thread" in t for t in trace)
    assert rec["lost"] == [1] and rec["epoch"] == 1
    assert rec["from"] == "fault" and rec["resumed_ms"] is not None
    assert rec["coordinator"]["pre_formed_groups"] == [0, 1]  # the cover group was adopted
    assert min(rec["coordinator"]["committed_tokens"]) > PROMPT  # resumed from restored decode rows
    assert mism == 0
    assert out == base, "streams differ from the no-fault run"
    assert all(len(o) == TOKENS for o in out)
    # the coordinator's view: epoch 1, the spare holds rank 1, no spare left standing
    st = view["status"]
    assert st["epoch"] == 1 and not st["down"] and st["spares"] == []
    conds = {c["type"]: c["status"] for c in st["conditions"]}
    assert conds["Ready"] == "True" and conds["Progressing"] == "False" and conds["Degraded"] == "True"
    assert sorted(w["rank"] for w in st["workers"]) == [0, 1]


@pytest.mark.slow
def test_loss_without_spare_abandons(tmp_path):
    from everserve_b200.serving.executor import EngineDown

    with pytest.raises(EngineDown):
        _run(tmp_path / "nospare", kill_at=3, spares=())


@pytest.mark.slow
def test_planned_departure_spare_catches_up(tmp_path):
    base, _, _, _ = _run(tmp_path / "nofault", spares=())
    cfg = EngineConfig(model=MODEL, device="cpu", dtype=torch.float32, num_blocks=128, max_batch=STREAMS,
                       max_model_len=PROMPT + TOKENS + 16, pipeline_parallel=2, use_cuda_graphs=False)
    with ControlPlane(str(tmp_path / "drain"), engines=[{"name": "e0", "pipelineParallel": 2}]) as cp:
        ex = MultiprocExecutor(cfg, engine="e0", daemon=cp.daemon_socket, store=cp.store_socket, spares=(1,),
                               node="n0", log_dir=str(tmp_path / "drain" / "logs"), threads=2)
        try:
            cp.wait_spares("e0", 1)
            eng = Engine(cfg, executor=ex)
            eng.wrap_step(failover(ex, eng))
            ex.notice_at_decode_step = (10, 1)
            out = eng.generate(_prompts(), max_tokens=TOKENS)
            assert len(ex.changes) == 1 and ex.changes[0].lost == [1]
            assert out == base
            # the departing rank left cleanly (released, exit 0)
            assert ex.procs["rank1"].wait(timeout=30) == 0
        finally:
            ex.shutdown()


@pytest.mark.slow
def test_daemon_launched_spare_replays_startup_and_takes_over(tmp_path):
    """The policy places a spare for rank 1 on n0; the daemon launches it, it fetches the
    engine's start-up record from the head (ReplayAsk/ReplayOffer), stands, and takes rank 1
    after rank 1 is killed. A spare that exits before any fault is started again."""
    import sys
    import time

    base, _, _, _ = _run(tmp_path / "nofault", spares=())
    cfg = EngineConfig(model=MODEL, device="cpu", dtype=torch.float32, num_blocks=128, max_batch=STREAMS,
                       max_model_len=PROMPT + TOKENS + 16, pipeline_parallel=2, use_cuda_graphs=False)
    engines = [{"name": "e0", "pipelineParallel": 2, "spares": [{"node": "n0", "device": 0, "rank": 1}],
                "spareLaunch": {"command": [sys.executable, "-m", "everserve_b200.serving.spare"],
                                "env": {"PYTHONPATH": os.path.dirname(os.path.dirname(os.path.abspath(__file__)))}}}]
    with ControlPlane(str(tmp_path / "launched"), engines=engines) as cp:
        ex = MultiprocExecutor(cfg, engine="e0", daemon=cp.daemon_socket, store=cp.store_socket, spares=(),
                               node="n0", log_dir=str(tmp_path / "launched" / "logs"), threads=2)
        try:
            cp.wait_spares("e0", 1, timeout_s=300)
            # supervision: the standing spare is killed; the daemon starts another
            first = cp.engine_view("e0")["status"]["spares"]
            import signal as sig

            pid = int(open(os.path.join(cp.dir, "node.log")).read().split("(pid ")[1].split(",")[0])
            os.kill(pid, sig.SIGKILL)
            deadline = time.monotonic() + 120
            while time.monotonic() < deadline:
                log = open(os.path.join(cp.dir, "node.log")).read()
                if "start 2)" in log and cp.engine_view("e0")["status"]["spares"]:
                    break
                time.sleep(0.2)
            assert "start 2)" in open(os.path.join(cp.dir, "node.log")).read()
            assert first
            _wait_covered(cp, "e0")
            eng = Engine(cfg, executor=ex)
            eng.wrap_step(failover(ex, eng))
            ex.kill_at_decode_step = (KILL_AT, 1)
            out = eng.generate(_prompts(), max_tokens=TOKENS)
            assert len(ex.changes) == 1 and out == base
        finally:
            ex.shutdown()


@pytest.mark.slow
def test_coordinator_dies_mid_change_standby_finishes_it(tmp_path):
    """The active coordinator logs the change to the spec store and dies before any node hears of
    it; the standby takes the lease, reads the log, waits for the daemon to link again and
    finishes the change. The streams stay token-identical."""
    base, _, _, _ = _run(tmp_path / "nofault", spares=())
    cfg = EngineConfig(model=MODEL, device="cpu", dtype=torch.float32, num_blocks=128, max_batch=STREAMS,
                       max_model_len=PROMPT + TOKENS + 16, pipeline_parallel=2, use_cuda_graphs=False)
    with ControlPlane(str(tmp_path / "takeover"), engines=[{"name": "e0", "pipelineParallel": 2}], standby=True,
                      coord_env={"EVERSERVE_COORD_EXIT_AFTER_LOG": "1"}) as cp:
        ex = MultiprocExecutor(cfg, engine="e0", daemon=cp.daemon_socket, store=cp.store_socket, spares=(1,),
                               node="n0", log_dir=str(tmp_path / "takeover" / "logs"), threads=2)
        try:
            cp.wait_spares("e0", 1)
            eng = Engine(cfg, executor=ex)
            eng.wrap_step(failover(ex, eng))
            ex.kill_at_decode_step = (KILL_AT, 1)
            out = eng.generate(_prompts(), max_tokens=TOKENS)
            assert cp.procs["coord"].poll() == 17  # the first coordinator died after logging
            assert "finishing it" in cp.log("coord-standby")
            assert len(ex.changes) == 1 and out == base
            assert cp.engine_view("e0")["status"]["epoch"] == 1
        finally:
            ex.shutdown()


@pytest.mark.slow
def test_spare_on_another_node_restores_from_its_replica(tmp_path):
    """Ranks on n0, the spare for rank 1 on n1 with its own daemon and store. The coordinator has
    n0's store replicate rank 1's rows to n1's store (a snapshot, then every commit); after rank 1
    is killed the spare restores from its own node's store and the streams stay identical."""
    base, _, _, _ = _run(tmp_path / "nofault", spares=())
    cfg = EngineConfig(model=MODEL, device="cpu", dtype=torch.float32, num_blocks=128, max_batch=STREAMS,
                       max_model_len=PROMPT + TOKENS + 16, pipeline_parallel=2, use_cuda_graphs=False)
    with ControlPlane(str(tmp_path / "two"), engines=[{"name": "e0", "pipelineParallel": 2}],
                      extra_nodes=["n1"]) as cp:
        place = {"daemon": cp.daemon_sockets["n1"], "store": cp.store_sockets["n1"], "node": "n1"}
        ex = MultiprocExecutor(cfg, engine="e0", daemon=cp.daemon_socket, store=cp.store_socket, spares=(1,),
                               node="n0", log_dir=str(tmp_path / "two" / "logs"), threads=2, spare_places=[place])
        try:
            cp.wait_spares("e0", 1)
            _wait_covered(cp, "e0")
            eng = Engine(cfg, executor=ex)
            eng.wrap_step(failover(ex, eng))
            ex.kill_at_decode_step = (KILL_AT, 1)
            out = eng.generate(_prompts(), max_tokens=TOKENS)
            assert len(ex.changes) == 1 and out == base
            # the spare resumed from rows it restored (decode positions), not from a re-prefill
            committed = ex.changes[0].coordinator["committed_tokens"]
            assert min(committed) > PROMPT, ex.changes[0].coordinator
            view = cp.engine_view("e0")["status"]
            assert {w["rank"]: w["node"] for w in view["workers"]} == {0: "n0", 1: "n1"}
            assert "replicates e0:1" in cp.log("node")
        finally:
            ex.shutdown()


@pytest.mark.slow
def test_node_agent_starts_remote_ranks(tmp_path):
    """The head starts rank 0 on n0; a node agent on n1 fetches the start-up record through the
    control plane and starts rank 1 there. The two-node engine serves the same tokens."""
    import subprocess
    import sys

    base, _, _, _ = _run(tmp_path / "nofault", spares=())
    cfg = EngineConfig(model=MODEL, device="cpu", dtype=torch.float32, num_blocks=128, max_batch=STREAMS,
                       max_model_len=PROMPT + TOKENS + 16, pipeline_parallel=2, use_cuda_graphs=False)
    with ControlPlane(str(tmp_path / "agents"), engines=[{"name": "e0", "pipelineParallel": 2}],
                      extra_nodes=["n1"]) as cp:
        env = dict(os.environ, EVERSERVE_SOCKET=cp.daemon_sockets["n1"], EVERSERVE_MIRROR_SOCKET=cp.store_sockets["n1"],
                   EVERSERVE_NODE="n1", PYTHONPATH=os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
        agent = subprocess.Popen([sys.executable, "-m", "everserve_b200.serving.node", "--engine", "e0", "--ranks", "1",
                                  "--threads", "2"], env=env)
        ex = MultiprocExecutor(cfg, engine="e0", daemon=cp.daemon_socket, store=cp.store_socket, spares=(),
                               node="n0", log_dir=str(tmp_path / "agents" / "logs"), threads=2, local_ranks=[0])
        try:
            out = Engine(cfg, executor=ex).generate(_prompts(), max_tokens=TOKENS)
            assert out == base
            view = cp.engine_view("e0")["status"]
            assert {w["rank"]: w["node"] for w in view["workers"]} == {0: "n0", 1: "n1"}
        finally:
            ex.shutdown()
            assert agent.wait(timeout=60) == 0


@pytest.mark.slow
def test_sampled_streams_replay_exactly_after_sigkill(tmp_path):
    """Temperature / top-p / top-k sampling with a seed: the resumed streams draw what the lost
    rank's steps drew (the draw is a function of seed and position), so they finish identical."""
    kw = dict(temperature=0.8, top_p=0.95, top_k=40, seed=5)
    base, _, _, _ = _run(tmp_path / "nofault", spares=(), **kw)
    greedy, _, _, _ = _run(tmp_path / "greedy", spares=())
    assert base != greedy
    out, changes, mism, _ = _run(tmp_path / "fault", kill_at=KILL_AT, **kw)
    assert len(changes) == 1 and mism == 0
    assert out == base


def test_logprobs_through_the_multiprocess_engine(tmp_path):
    """Log-probabilities come back from the last stage's ranks and match a single process's."""
    from everserve_b200.engine.request import SamplingParams

    cfg = EngineConfig(model=MODEL, device="cpu", dtype=torch.float32, num_blocks=128, max_batch=STREAMS,
                       max_model_len=PROMPT + TOKENS + 16, pipeline_parallel=2, use_cuda_graphs=False)
    prompts = _prompts()[:2]
    sp = SamplingParams(max_tokens=4, logprobs=2)
    one = Engine(EngineConfig(model=MODEL, device="cpu", dtype=torch.float32, num_blocks=128, max_batch=STREAMS,
                              max_model_len=PROMPT + TOKENS + 16, use_cuda_graphs=False))
    ids1 = [one.add_request(p, sp) for p in prompts]
    while one.has_work():
        one.step()
    with ControlPlane(str(tmp_path / "cp"), engines=[{"name": "e0", "pipelineParallel": 2}]) as cp:
        ex = MultiprocExecutor(cfg, engine="e0", daemon=cp.daemon_socket, store=cp.store_socket, spares=(),
                               node="n0", log_dir=str(tmp_path / "logs"), threads=2)
        try:
            eng = Engine(cfg, executor=ex)
            ids = [eng.add_request(p, sp) for p in prompts]
            while eng.has_work():
                eng.step()
            for a, b in zip(ids, ids1):
                ra, rb = eng.request(a), one.request(b)
                assert ra.outputs == rb.outputs and len(ra.logprobs) == 4
                for (la, ta), (lb, tb) in zip(ra.logprobs, rb.logprobs):
                    assert abs(la - lb) < 1e-4 and [t for t, _ in ta] == [t for t, _ in tb]
        finally:
            ex.shutdown()


@pytest.mark.slow
def test_rank_killed_during_prefill_is_replaced_and_prefill_runs_again(tmp_path):
    """Nothing is committed when a rank dies in the middle of the first prefill: every request
    goes back to the queue and is prefilled again on the new membership."""
    base, _, _, _ = _run(tmp_path / "nofault", spares=())
    out, changes, mism, _ = _run(tmp_path / "fault", kill_prefill=(1, 1))
    assert len(changes) == 1 and changes[0].lost == [1]
    assert mism == 0 and out == base


@pytest.mark.slow
def test_two_ranks_killed_at_once_both_replaced(tmp_path):
    """Both stages lose their process in the same step; a spare stands for each and both take
    their ranks in one change."""
    base, _, _, _ = _run(tmp_path / "nofault", spares=())
    out, changes, mism, view = _run(tmp_path / "fault", kill_at=(KILL_AT, [0, 1]), spares=(0, 1))
    assert len(changes) == 1 and sorted(changes[0].lost) == [0, 1]
    assert mism == 0 and out == base
    assert view["status"]["epoch"] == 1
