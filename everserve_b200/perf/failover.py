"""Failover latency: dead-rank detection, change commit, resume and the streams' pause.

    python -m everserve_b200.perf.failover [--trials 20] [--model tiny-qwen] [--full] [--device cpu]
                                           [--tp 1 --pp 2] [--streams 8] [--victim R]

Each trial starts the control plane (coordinator, daemon, store) and an engine (TP1 PP2 by
default; ``--tp 2 --pp 1`` for the tensor-parallel group whose collectives detect the loss;
``--tp 1 --pp 1`` for a one-rank engine, whose rank 0 leaves: ``--victim`` picks the rank) with a
spare for the victim rank (rank 1 by default), generates the streams, kills the victim at a random
decode step (SIGKILL on the CPU
tier; between steps on GPUs, where the spare sits on the GPU after the engine's) and checks every
stream against a no-fault run. Per trial it records, from the fault (the coordinator's stamps are
wall-clock microseconds of the same host):

  * detect_ms   - the coordinator received the loss (its ``reported_at_us``);
  * commit_ms   - the coordinator committed the new membership;
  * resumed_ms  - the head resumed the engine (groups formed, requests restarted);
  * pause_ms    - the longest gap between two steps that produced tokens, around the fault: what a
                  client of the streams sees;
  * tok_s_before / tok_s_after - the streams' decode tokens per second (wall clock, through the
                  engine's public step) over the steps before the fault and after the resume.

It prints one JSON line with p50 / p99 / max of each and the token-identity verdict.
``--full`` uses the Qwen2.5-0.5B shape (128-token prompts, 64 tokens, kill at decode step 20).
"""

from __future__ import annotations

import argparse
import json
import os
import random
import shutil
import tempfile
import time

import torch


def _pct(xs, q):
    xs = sorted(xs)
    if not xs:
        return None
    k = min(len(xs) - 1, max(0, int(round(q / 100 * (len(xs) - 1)))))
    return round(xs[k], 3)


def _rate(stamps):
    """Tokens per second over consecutive (time, tokens) stamps: the tokens after the first stamp
    over the time since it."""
    if len(stamps) < 2:
        return None
    dt = stamps[-1][0] - stamps[0][0]
    return round(sum(n for _, n in stamps[1:]) / dt, 1) if dt > 0 else None


def run_trial(workdir, model, prompts, tokens, kill_at, device, dtype, tp=1, pp=2, victim=1):
    from ..engine.config import EngineConfig
    from ..engine.engine import Engine
    from ..serving.cluster import ControlPlane
    from ..serving.executor import MultiprocExecutor, failover

    cfg = EngineConfig(model=model, device=device, dtype=dtype, num_blocks=256, max_batch=len(prompts),
                       max_model_len=len(prompts[0]) + tokens + 16, pipeline_parallel=pp,
                       tensor_parallel=tp, use_cuda_graphs=False)
    gpu = device.startswith("cuda")
    # GPU failure tests keep NCCL's NVLS and the kernels' multicast variant off
    env = {"NCCL_NVLS_ENABLE": "0", "ES_NVLS": "0", "EVERSERVE_DETECT_FLOOR_MS": "20"} if gpu else None
    with ControlPlane(workdir, engines=[{"name": "e0", "pipelineParallel": pp, "tensorParallel": tp}]) as cp:
        ex = MultiprocExecutor(cfg, engine="e0", daemon=cp.daemon_socket, store=cp.store_socket,
                               spares=(victim,) if kill_at else (), node="n0", threads=2,
                               device="cuda" if gpu else "cpu", dtype="bfloat16" if gpu else "float32",
                               env=env)
        try:
            if kill_at:
                cp.wait_spares("e0", 1)
            eng = Engine(cfg, executor=ex)
            eng.wrap_step(failover(ex, eng))
            if kill_at:
                ex.kill_at_decode_step = (kill_at, victim)
            from ..engine.request import SamplingParams

            ids = [eng.add_request(p, SamplingParams(max_tokens=tokens)) for p in prompts]
            stamps = []
            while eng.has_work():
                out = eng.step()
                n = sum(1 for _, tok, _ in out if tok is not None)
                if n:
                    stamps.append((time.monotonic(), n))
            outs = [eng.request(i).outputs for i in ids]
            rec = ex.changes[0] if ex.changes else None
            return outs, rec, stamps
        finally:
            ex.shutdown()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--trials", type=int, default=10)
    ap.add_argument("--model", default="tiny-qwen")
    ap.add_argument("--full", action="store_true", help="Qwen2.5-0.5B shape, 128-token prompts, 64 tokens")
    ap.add_argument("--device", default="cpu")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--pp", type=int, default=2)
    ap.add_argument("--streams", type=int, default=8)
    ap.add_argument("--victim", type=int, default=None,
                    help="the rank that leaves (default 1; 0 for a one-rank engine, --tp 1 --pp 1)")
    a = ap.parse_args()
    victim = a.victim if a.victim is not None else (1 if a.tp * a.pp > 1 else 0)
    assert 0 <= victim < a.tp * a.pp, "the victim must be a rank of the engine"
    model = "qwen2.5-0.5b" if a.full else a.model
    from ..models.config import get_config

    vocab = get_config(model).vocab
    prompt_len, tokens = (128, 64) if a.full else (64, 32)
    rng = random.Random(a.seed)
    prompts = [[rng.randrange(vocab) for _ in range(prompt_len)] for _ in range(a.streams)]
    dtype = torch.bfloat16 if a.device.startswith("cuda") else torch.float32
    root = tempfile.mkdtemp(prefix="es-failover-")
    try:
        base, _, base_stamps = run_trial(os.path.join(root, "base"), model, prompts, tokens, 0, a.device, dtype,
                                         a.tp, a.pp, victim)
        rows = []
        for t in range(a.trials):
            kill_at = 20 if a.full else rng.randrange(3, tokens - 4)
            outs, rec, stamps = run_trial(os.path.join(root, f"t{t}"), model, prompts, tokens, kill_at, a.device,
                                          dtype, a.tp, a.pp, victim)
            d = rec.as_dict()
            t_fault = rec.t_fault_wall
            rep_us = rec.coordinator.get("reported_at_us")
            times = [ts for ts, _ in stamps]
            gaps = [b - a_ for a_, b in zip(times, times[1:])]
            cut = max(range(len(gaps)), key=lambda i: gaps[i]) if gaps else 0
            rows.append({
                "kill_at": kill_at, "identical": outs == base,
                "detect_ms": (rep_us / 1e3 - t_fault * 1e3) if rep_us else None,
                "commit_ms": d["committed_ms"], "resumed_ms": d["resumed_ms"],
                "pause_ms": max(gaps) * 1e3 if gaps else None,
                "tok_s_before": _rate(stamps[1:cut + 1]), "tok_s_after": _rate(stamps[cut + 2:]),
                "spans": d["spans"], "acks_at_us": rec.coordinator.get("acks_at_us"),
            })
        summary = {"metric": "failover pause p99; dead-rank detect ms", "model": model, "device": a.device,
                   "tp": a.tp, "pp": a.pp, "victim": victim, "streams": a.streams, "trials": len(rows),
                   "token_identical": all(r["identical"] for r in rows),
                   "tok_s_no_fault": _rate(base_stamps[1:])}
        for k in ("detect_ms", "commit_ms", "resumed_ms", "pause_ms", "tok_s_before", "tok_s_after"):
            xs = [r[k] for r in rows if r[k] is not None]
            summary[k] = {"p50": _pct(xs, 50), "p99": _pct(xs, 99), "max": round(max(xs), 3) if xs else None}
        summary["rows"] = rows
        print(json.dumps(summary))
    finally:
        shutil.rmtree(root, ignore_errors=True)


if __name__ == "__main__":
    main()
