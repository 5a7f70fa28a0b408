"""In-kernel detection of a member that stops, on the GPUs of one node (one process per GPU).

    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 \\
        -m everserve_b200.perf.detect [--trials 5] [--beat-limit-ms 20] [--elems 4096]

Every rank builds the failure-detecting collective (peer stores into driver VMM buffers; NVLS off,
as every failure test here) with a beat limit. The members run decode-size all-reduces in lock-step
(each rank's calls back to back on its stream); at a random call the last rank stops: it stops its
heartbeat thread and enters no more calls. It stops between two calls, after synchronizing, so
none of its kernels is in flight: the fault is made on the host. The other members' next call must
end on its own with the dead status naming that member, within the beat limit, not the hard limit.

Per trial, on each surviving rank: the device time of the call that detected the loss (CUDA events
around it: from its launch to its return, which is what a decode step would wait), the status and
the late mask it left, and the device time of a healthy call for scale. Then every member resumes
(call counters and buffers zeroed, the heartbeat restarted) and the next trial starts. Rank 0
prints one JSON line per trial and a summary.
"""

from __future__ import annotations

import argparse
import json
import os
import random
import time
from datetime import timedelta

import torch
import torch.distributed as dist

DEAD = 4


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--trials", type=int, default=5)
    ap.add_argument("--beat-limit-ms", type=float, default=20.0)
    ap.add_argument("--elems", type=int, default=4096)
    ap.add_argument("--seed", type=int, default=0)
    a = ap.parse_args()
    os.environ.setdefault("ES_NVLS", "0")
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    rank, world = dist.get_rank(), dist.get_world_size()
    if world < 2:
        raise SystemExit("needs 2 or more ranks")
    from ..parallel.fused import BEAT_PERIOD_US, FusedTPCollective

    coll = FusedTPCollective(dev, group=dist.group.WORLD, nvls=False)
    coll.set_beat_limit_us(int(a.beat_limit_ms * 1000))
    coll.set_bound_ns(10_000_000_000)  # the hard bound far away: the beat must name the member
    x = torch.ones(a.elems, dtype=torch.bfloat16, device=dev)
    out = torch.empty_like(x)
    rng = random.Random(a.seed)
    stopper = world - 1
    rows = []

    def timed_call():
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        coll.all_reduce_into(x, out)
        e.record()
        torch.cuda.synchronize()
        return s.elapsed_time(e)

    for t in range(a.trials):
        stop_at = rng.randrange(5, 50)
        # healthy calls in lock-step (the last one timed for scale)
        healthy = 0.0
        for i in range(stop_at):
            healthy = timed_call()
        ok_before = coll.status() == 0 and bool((out.float() == world).all())
        detect_ms, status, late = None, None, None
        if rank == stopper:
            # leave between calls: nothing in flight, then stand still
            torch.cuda.synchronize()
            coll.C.heartbeat_stop(coll._beat)
            coll._beat = 0
        else:
            detect_ms = timed_call()
            status, late = coll.status(), coll.late_rows()
        # every rank is idle now; meet on the host store (no device collective)
        _store_barrier(t, rank, world)
        if rank == stopper:
            coll._beat = int(coll.C.heartbeat_start(coll.region.beat_address(coll.row), BEAT_PERIOD_US))
        coll.resume()
        _store_barrier(1000 + t, rank, world)
        res = torch.tensor([detect_ms or 0.0, float(status or 0), float(sum(1 << r for r in (late or []))),
                            healthy * 1e3, float(ok_before)], dtype=torch.float64, device=dev)
        allr = [torch.zeros_like(res) for _ in range(world)]
        dist.all_gather(allr, res)
        if rank == 0:
            surv = [r.tolist() for i, r in enumerate(allr) if i != stopper]
            row = {"trial": t, "stop_after_calls": stop_at, "stopped_rank": stopper,
                   "detect_ms": [round(s[0], 3) for s in surv],
                   "status": [int(s[1]) for s in surv], "late_mask": [int(s[2]) for s in surv],
                   "healthy_call_us": round(max(s[3] for s in surv), 2),
                   "results_exact_before": all(bool(s[4]) for s in surv)}
            row["named_dead"] = all(s == DEAD for s in row["status"]) and all(m == 1 << stopper
                                                                              for m in row["late_mask"])
            rows.append(row)
            print(json.dumps(row), flush=True)
    if rank == 0:
        det = sorted(d for r in rows for d in r["detect_ms"])
        print(json.dumps({"metric": "in-kernel dead-member detection", "n_gpus": world, "trials": len(rows),
                          "beat_limit_ms": a.beat_limit_ms, "beat_period_us": BEAT_PERIOD_US,
                          "all_named_dead": all(r["named_dead"] for r in rows),
                          "detect_ms_p50": det[len(det) // 2] if det else None,
                          "detect_ms_max": det[-1] if det else None,
                          "healthy_call_us_max": max(r["healthy_call_us"] for r in rows) if rows else None}),
              flush=True)
    torch.cuda.synchronize()
    _store_barrier(99999, rank, world)
    coll.close()
    dist.destroy_process_group()


def _store_barrier(tag: int, rank: int, world: int) -> None:
    """A barrier over the rendezvous store (host only: no kernel, no NCCL call)."""
    store = dist.distributed_c10d._get_default_store()
    store.add(f"es_detect_{tag}", 1)
    t0 = time.monotonic()
    while int(store.add(f"es_detect_{tag}", 0)) < world:
        if time.monotonic() - t0 > 120:
            raise TimeoutError(f"store barrier {tag}")
        time.sleep(0.001)


if __name__ == "__main__":
    main()
