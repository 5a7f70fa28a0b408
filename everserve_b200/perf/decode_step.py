"""Time one decode step of a model with a synthetic KV history (no prefill needed).

    python -m everserve_b200.perf.decode_step --model llama-3-8b --batch 64 --ctx 1024 --steps 20

The KV cache holds ``ctx`` random positions per sequence; each step decodes one token per sequence
through the same model forward the engine captures (a CUDA graph unless ``--eager``). ``--layers``
narrows the model for small profiler captures. Times are CUDA-event times per step (max over
ranks). Under torchrun the model is tensor-parallel over the ranks (``--collective fused|nccl``).
``--breakdown`` adds per-kernel device time of one eager step from a CUPTI trace (torch.profiler);
those times are for attribution only, the step time above is measured without the tracer.
"""

from __future__ import annotations

import argparse
import dataclasses
import json

import torch

from ..models.config import get_config
from ..models.llama import DecoderLM, StepInput


def build(model: str, batch: int, ctx: int, layers: int | None, bs: int = 16, seed: int = 0, tp=None):
    cfg = get_config(model)
    if layers:
        cfg = dataclasses.replace(cfg, layers=layers)
    dev = torch.device("cuda", torch.cuda.current_device())
    m = DecoderLM(cfg, dev, torch.bfloat16, seed, tp=tp)
    max_len = ctx + 64
    mb = (max_len + bs - 1) // bs
    nb = batch * mb
    g = torch.Generator(device=dev).manual_seed(seed)
    caches = [torch.randn(m.kv_cache_shape(nb, bs), generator=g, device=dev).bfloat16() for _ in range(cfg.layers)]
    bt = torch.arange(nb, device=dev, dtype=torch.int32).view(batch, mb)
    pos = torch.full((batch,), ctx, device=dev, dtype=torch.int64)
    slots = bt[:, ctx // bs].long() * bs + ctx % bs
    ids = torch.randint(0, cfg.vocab, (batch,), device=dev, generator=g)
    inp = StepInput(ids=ids, positions=pos, slots=slots, block_tables=bt,
                    ctx_lens=(pos + 1).int(), q_seq=torch.arange(batch, device=dev), logits_idx=torch.arange(batch, device=dev),
                    is_decode=True, max_model_len=max_len)
    m.ops.reserve_linear(batch, m.linear_shapes())
    m.ops.reserve_attention(batch, m.hq, m.d, max_len)
    return m, caches, inp


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="llama-3-8b")
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--ctx", type=int, default=1024)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--layers", type=int, default=None)
    ap.add_argument("--eager", action="store_true")
    ap.add_argument("--collective", default="fused", choices=["fused", "nccl"])
    ap.add_argument("--breakdown", action="store_true")
    a = ap.parse_args()
    import os

    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    tp = None
    coll = None
    if world > 1:
        from datetime import timedelta

        from ..models.llama import TPGroup
        from ..parallel.collective import make_tp_collective

        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local), timeout=timedelta(seconds=120))
        coll = make_tp_collective(torch.device("cuda", local), kind=a.collective)
        tp = TPGroup(rank, world, coll)
    m, caches, inp = build(a.model, a.batch, a.ctx, a.layers, tp=tp)
    fwd = lambda: m.forward(inp, caches)  # noqa: E731
    for _ in range(2):
        fwd()
    torch.cuda.synchronize()
    run = fwd
    if not a.eager:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fwd()
        run = g.replay
        run()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(a.steps):
        run()
    end.record()
    torch.cuda.synchronize()
    ms = start.elapsed_time(end) / a.steps
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    w_bytes = sum(w.numel() * w.element_size() for w in m.weights.values())
    kv_bytes = a.batch * (a.ctx + 1) * 2 * m.hkv * m.d * 2 * (m.l1 - m.l0)
    if rank != 0:
        pass
    else:
        print(json.dumps({"model": a.model, "layers": m.l1 - m.l0, "batch": a.batch, "ctx": a.ctx, "ms_per_step": round(ms, 4),
                      "tok_s": round(a.batch / ms * 1e3, 1), "weight_gb": round(w_bytes / 1e9, 3),
                      "kv_gb": round(kv_bytes / 1e9, 3), "gb_s": round((w_bytes + kv_bytes) / ms / 1e6, 1),
                      "status": m.ops.check_status(), "tp": world}))
    if a.breakdown:
        breakdown(fwd, rank)
    del run
    if not a.eager:
        del g
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        if coll is not None and hasattr(coll, "close"):
            coll.close()
        dist.destroy_process_group()


def breakdown(fwd, rank: int) -> None:
    from torch.profiler import ProfilerActivity, profile

    fwd()
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fwd()
        torch.cuda.synchronize()
    agg: dict[str, list[float]] = {}
    for e in prof.key_averages():
        us = getattr(e, "self_device_time_total", 0) or getattr(e, "self_cuda_time_total", 0)
        if us > 0:
            name = e.key.split("(")[0][:60]
            v = agg.setdefault(name, [0.0, 0])
            v[0] += us
            v[1] += e.count
    if rank == 0:
        total = sum(v[0] for v in agg.values())
        for name, (us, n) in sorted(agg.items(), key=lambda kv: -kv[1][0])[:25]:
            print(json.dumps({"kernel": name, "us": round(us, 1), "calls": n, "share": round(us / total, 3)}))
        print(json.dumps({"kernel": "TOTAL", "us": round(total, 1)}))


if __name__ == "__main__":
    main()
