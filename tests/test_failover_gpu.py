"""Failover on GPUs: a tensor-parallel engine loses a rank and a spare on another GPU takes it.

TP2 on GPUs 0-1 plus a spare for rank 1 on GPU 2, with the C++ coordinator, node daemon and KV
store. The row-parallel linears run the fused GEMM + all-reduce kernel over peer memory (driver VMM
buffers, plain peer stores; NVLS off), every wait bounded. Rank 1 leaves between two decode steps
(nothing of it in flight); rank 0's next collective waits out its bound, names rank 1 late, and its
SlotWatch finds the process dead, raises the abort word and reports the loss. The coordinator
replaces rank 1 with the spare, which restores rank 1's committed KV with the scatter kernel; the
survivor re-points its member table at the spare's buffer (no communicator is rebuilt), and every
stream completes token-identical to the no-fault run.

Needs 3 GPUs (skipped otherwise). A second test needs 2: a one-rank engine on GPU 0 whose rank
leaves, and a spare on GPU 1 that takes it (no collective; the store restore and the resume).
"""

import os
import random

import pytest
import torch

pytestmark = pytest.mark.gpu

STREAMS, PROMPT, TOKENS, KILL_AT, MODEL = 4, 48, 24, 6, "small-llama"


def _run(workdir, kill_at=None, spares=(1,), tp=2, victim=1):
    from everserve_b200.engine.config import EngineConfig
    from everserve_b200.engine.engine import Engine
    from everserve_b200.serving.cluster import ControlPlane
    from everserve_b200.serving.executor import MultiprocExecutor, failover

    rng = random.Random(0)
    prompts = [[rng.randrange(4096) for _ in range(PROMPT)] for _ in range(STREAMS)]
    cfg = EngineConfig(model=MODEL, device="cuda", dtype=torch.bfloat16, num_blocks=64, max_batch=STREAMS,
                       max_model_len=PROMPT + TOKENS + 16, tensor_parallel=tp, use_cuda_graphs=False)
    env = {"NCCL_NVLS_ENABLE": "0", "ES_NVLS": "0", "EVERSERVE_DETECT_FLOOR_MS": "20"}
    with ControlPlane(str(workdir), engines=[{"name": "g0", "tensorParallel": tp}]) as cp:
        ex = MultiprocExecutor(cfg, engine="g0", daemon=cp.daemon_socket, store=cp.store_socket, spares=spares,
                               node="n0", device="cuda", dtype="bfloat16", env=env, log_dir=str(workdir / "logs"),
                               step_timeout_s=120, change_timeout_s=120)
        try:
            if spares:
                cp.wait_spares("g0", len(spares), timeout_s=300)
            eng = Engine(cfg, executor=ex)
            eng.wrap_step(failover(ex, eng))
            if kill_at is not None:
                ex.kill_at_decode_step = (kill_at, victim)
            out = eng.generate(prompts, max_tokens=TOKENS)
            mism = sum(r.replay_mismatches for r in eng.scheduler.requests.values())
            return out, [c.as_dict() for c in ex.changes], mism
        finally:
            ex.shutdown()


def test_tp2_rank_loss_spare_takes_over_token_identical(tmp_path):
    if torch.cuda.device_count() < 3:
        pytest.skip("needs 3 GPUs")
    base, _, _ = _run(tmp_path / "nofault", spares=())
    out, changes, mism = _run(tmp_path / "fault", kill_at=KILL_AT)
    print("change:", changes)
    assert len(changes) == 1 and changes[0]["lost"] == [1]
    assert mism == 0
    assert out == base
    out_dir = os.environ.get("ES_RESULTS_DIR")
    if out_dir:  # keep the change's timeline when asked to
        os.makedirs(out_dir, exist_ok=True)
        with open(os.path.join(out_dir, "failover_gpu.txt"), "a") as f:
            f.write(f"{changes}\n")


def test_tp1_rank_loss_spare_on_another_gpu_token_identical(tmp_path):
    """Two GPUs: the only rank (GPU 0) leaves between decode steps; the spare on GPU 1 restores its
    committed KV from the store (through the pinned copy: the store lives on the temporary
    directory's filesystem) and every stream completes token-identical."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    base, _, _ = _run(tmp_path / "nofault", spares=(), tp=1)
    out, changes, mism = _run(tmp_path / "fault", kill_at=KILL_AT, spares=(0,), tp=1, victim=0)
    print("change:", changes)
    assert len(changes) == 1 and changes[0]["lost"] == [0]
    assert mism == 0
    assert out == base
    out_dir = os.environ.get("ES_RESULTS_DIR")
    if out_dir:
        os.makedirs(out_dir, exist_ok=True)
        with open(os.path.join(out_dir, "failover_gpu_tp1.txt"), "a") as f:
            f.write(f"{changes}\n")

