"""Collective microbenchmark (the failure-detecting all-reduce configuration) on the GPUs of one node, one process per GPU.

    python -m torch.distributed.run --nproc-per-node N -m everserve_b200.perf.collectives [--sizes ...]

For bf16 tensors of 4 KiB .. 256 MiB (powers of two; values N(0,1) from the seed):
  * fdar: the failure-detecting all-reduce over peer memory (LL protocol for small tensors, two-shot
    above; tensors above one call's capacity in several calls),
  * nccl: torch.distributed.all_reduce,
timed as a CUDA graph of `iters` back-to-back calls (device time, max over ranks), reported as
bus bandwidth 2 (n - 1) / n * bytes / time. Then the row-parallel GEMM + all-reduce at the
configuration's shape [4096 x K] . [K x 4096] (K = 4096 / N: row blocks overlapped with their
all-reduces) and at the decode shape [64 x K] . [K x 4096] (K = 4096 / N, and the 8B model's down
projection K = 14336 / N: one fused kernel), each against the same GEMM without the all-reduce and
against GEMM + NCCL.
"""

from __future__ import annotations

import argparse
import json
import os
from datetime import timedelta

import torch
import torch.distributed as dist


def graph_time(fn, iters: int) -> float:
    fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(iters):
            fn()
    g.replay()
    torch.cuda.synchronize()
    dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    g.replay()
    e.record()
    torch.cuda.synchronize()
    t = torch.tensor([s.elapsed_time(e) / iters], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    del g
    torch.cuda.synchronize()
    return float(t.item())


def eager_time(fn, iters: int) -> float:
    """Device time per call of `fn` run eagerly (work on side streams included), max over ranks."""
    fn()
    torch.cuda.synchronize()
    dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    t = torch.tensor([s.elapsed_time(e) / iters], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--min-bytes", type=int, default=4096)
    ap.add_argument("--max-bytes", type=int, default=256 << 20)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--skip-nccl-above", type=int, default=1 << 40)
    ap.add_argument("--variant", default="fused", choices=["fused", "p2p"])
    a = ap.parse_args()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    rank, world = dist.get_rank(), dist.get_world_size()
    from ..ops import KernelOps
    from ..parallel.collective import make_tp_collective

    coll = make_tp_collective(dev, kind=a.variant)
    kops = KernelOps(dev)
    rows = []
    nbytes = a.min_bytes
    while nbytes <= a.max_bytes:
        n = nbytes // 2
        g = torch.Generator(device="cuda").manual_seed(rank)
        x = torch.randn(n, generator=g, device=dev).bfloat16()
        bus = 2 * (world - 1) / world * nbytes
        row = {"bytes": nbytes, "n_gpus": world, "variant": coll.variant}
        # the failure-detecting kernels at every size (tensors above one call's capacity in calls)
        t = graph_time(lambda: coll.all_reduce_into(x, x), max(2, a.iters // (1 + nbytes // (64 << 20))))
        row.update(fdar_us=round(t * 1e3, 2), fdar_bus_gbs=round(bus / t / 1e6, 1))
        if nbytes <= a.skip_nccl_above:
            t = graph_time(lambda: dist.all_reduce(x), max(2, a.iters // (1 + nbytes // (64 << 20))))
            row.update(nccl_us=round(t * 1e3, 2), nccl_bus_gbs=round(bus / t / 1e6, 1))
        rows.append(row)
        nbytes *= 2
    # the configuration's fused variant: [4096 x K] . [K x 4096] with K = 4096 / N, the GEMM in row
    # blocks overlapped with the all-reduce of the block before, against GEMM + NCCL
    K = 4096 // world
    xm = torch.randn(4096, K, device=dev).bfloat16()
    w = (torch.randn(4096, K, device=dev) / 64).bfloat16()
    out = torch.empty(4096, 4096, device=dev, dtype=torch.bfloat16)
    t_fused = eager_time(lambda: coll.linear_allreduce(kops, xm, w), 10)
    t_gemm = eager_time(lambda: kops.linear(xm, w, out=out), 10)

    def unfused_big():
        y = kops.linear(xm, w, out=out)
        dist.all_reduce(y)

    t_nccl = eager_time(unfused_big, 10)
    rows.append({"fused_gemm_ar": f"[4096x{K}].[{K}x4096]", "n_gpus": world, "fused_us": round(t_fused * 1e3, 2),
                 "gemm_only_us": round(t_gemm * 1e3, 2), "gemm_plus_nccl_us": round(t_nccl * 1e3, 2),
                 "ar_bytes": 4096 * 4096 * 2})
    for K in (4096 // world, 14336 // world):
        xm = torch.randn(64, K, device=dev).bfloat16()
        w = (torch.randn(4096, K, device=dev) / 64).bfloat16()
        out = torch.empty(64, 4096, device=dev, dtype=torch.bfloat16)
        t_fused = graph_time(lambda: coll.linear_allreduce(kops, xm, w), a.iters)
        t_gemm = graph_time(lambda: kops.linear(xm, w, out=out), a.iters)

        def unfused():
            y = kops.linear(xm, w, out=out)
            dist.all_reduce(y)

        t_nccl = graph_time(unfused, a.iters)
        rows.append({"fused_gemm_ar": f"[64x{K}].[{K}x4096]", "n_gpus": world, "fused_us": round(t_fused * 1e3, 2),
                     "gemm_only_us": round(t_gemm * 1e3, 2), "gemm_plus_nccl_us": round(t_nccl * 1e3, 2)})
    if rank == 0:
        for r in rows:
            print(json.dumps(r), flush=True)
    torch.cuda.synchronize()
    dist.barrier()
    coll.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
