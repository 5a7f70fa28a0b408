"""Host-side cost of one decode step: scheduling, staging the inputs, applying the results.

    python -m everserve_b200.perf.host_step [--batch 64] [--prompt 1024] [--steps 200]

Everything the engine does on the CPU between two decode steps, without the model: the
scheduler's decode plan, the runner's staging of ids / positions / slots / block tables into the
pinned buffers, and the scheduler's update with the sampled ids. The GPU waits for this between
steps (the end-to-end number includes it), so it is kept to a small fraction of a step. Prints
one JSON line with microseconds per step for each part.
"""

from __future__ import annotations

import argparse
import json
import time

import torch


def measure(batch: int, prompt: int, steps: int) -> dict:
    from ..engine.block_manager import BlockManager
    from ..engine.request import Request, SamplingParams
    from ..engine.runner import ModelRunner
    from ..engine.scheduler import Scheduler

    bs, max_len = 16, prompt + steps + 64
    bm = BlockManager(batch * (max_len // bs + 2), bs)
    sch = Scheduler(bm, max_batch=batch, max_prefill_tokens=1 << 30, max_model_len=max_len)
    for _ in range(batch):
        sch.add(Request(list(range(prompt)), SamplingParams(max_tokens=steps + 32)))
    plan = sch.schedule()
    sch.update(plan, [1] * len(plan.reqs))

    runner = ModelRunner.__new__(ModelRunner)  # the staging half of a runner, no model
    runner.block_size, runner.max_batch, runner.max_model_len = bs, batch, max_len
    runner.max_blocks = (max_len + bs - 1) // bs
    runner.buckets = [b for b in (1, 2, 4, 8, 16, 24, 32, 48, 64, 96, 128, 192, 256) if b < batch] + [batch]
    runner.device = torch.device("cpu")
    runner.h_i64 = torch.zeros(4, batch, dtype=torch.int64)
    runner.h_bt = torch.zeros(batch, runner.max_blocks, dtype=torch.int32)
    runner.h_i64_np, runner.h_bt_np = runner.h_i64.numpy(), runner.h_bt.numpy()
    runner.d_i64, runner.d_bt = runner.h_i64.clone(), runner.h_bt.clone()
    runner._bt_rows = [(None, 0)] * batch
    runner.h_sf = torch.zeros(2, batch)
    runner.h_si = torch.zeros(2, batch, dtype=torch.int64)
    runner.d_sf, runner.d_si = runner.h_sf.clone(), runner.h_si.clone()

    t = {"schedule_us": 0.0, "stage_us": 0.0, "update_us": 0.0}
    ids = [5] * batch
    for _ in range(steps):
        t0 = time.perf_counter()
        plan = sch.schedule()
        t1 = time.perf_counter()
        runner.stage_decode(plan)
        t2 = time.perf_counter()
        sch.update(plan, ids[: len(plan.reqs)])
        t3 = time.perf_counter()
        t["schedule_us"] += t1 - t0
        t["stage_us"] += t2 - t1
        t["update_us"] += t3 - t2
    out = {k: round(v / steps * 1e6, 1) for k, v in t.items()}
    out["total_us"] = round(sum(out.values()), 1)
    return {"metric": "host work per decode step", "batch": batch, "context": prompt, **out}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--prompt", type=int, default=1024)
    ap.add_argument("--steps", type=int, default=200)
    a = ap.parse_args()
    print(json.dumps(measure(a.batch, a.prompt, a.steps)))


if __name__ == "__main__":
    main()
