"""Time one decode step of a model with a synthetic KV history (no prefill needed).

    python -m everserve_b200.perf.decode_step --model llama-3-8b --batch 64 --ctx 1024 --steps 20

The KV cache holds ``ctx`` random positions per sequence; each step decodes one token per sequence
through the same model forward the engine captures (a CUDA graph unless ``--eager``). ``--layers``
narrows the model for small profiler captures. Times are CUDA-event times per step.
"""

from __future__ import annotations

import argparse
import dataclasses
import json

import torch

from ..models.config import get_config
from ..models.llama import DecoderLM, StepInput


def build(model: str, batch: int, ctx: int, layers: int | None, bs: int = 16, seed: int = 0):
    cfg = get_config(model)
    if layers:
        cfg = dataclasses.replace(cfg, layers=layers)
    dev = torch.device("cuda", torch.cuda.current_device())
    m = DecoderLM(cfg, dev, torch.bfloat16, seed)
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
    a = ap.parse_args()
    m, caches, inp = build(a.model, a.batch, a.ctx, a.layers)
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
    w_bytes = sum(w.numel() * w.element_size() for w in m.weights.values())
    kv_bytes = a.batch * (a.ctx + 1) * 2 * m.hkv * m.d * 2 * (m.l1 - m.l0)
    print(json.dumps({"model": a.model, "layers": m.l1 - m.l0, "batch": a.batch, "ctx": a.ctx, "ms_per_step": round(ms, 4),
                      "tok_s": round(a.batch / ms * 1e3, 1), "weight_gb": round(w_bytes / 1e9, 3),
                      "kv_gb": round(kv_bytes / 1e9, 3), "gb_s": round((w_bytes + kv_bytes) / ms / 1e6, 1),
                      "status": m.ops.check_status()}))


if __name__ == "__main__":
    main()
