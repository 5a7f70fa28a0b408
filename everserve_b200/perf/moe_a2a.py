"""Time of one routed mixture layer (dispatch, grouped expert GEMMs, combine) on one GPU.

    python -m everserve_b200.perf.moe_a2a [--members 4] [--tokens 64] [--hidden 4096]
                                         [--inter 14336] [--experts 8] [--top-k 2]

Plays every member of an expert-parallel group of ``--members`` on this GPU (``ExpertAllToAll.
emulated``: one launch carries the whole group's traffic between local buffers), so the number is
the group's work serialised on one device: every expert's weights are read once per layer, and
the dispatch and combine move each routed row twice. It prints the device time per layer (CUDA
events, after warm-up, a buffer larger than L2 written between timed layers), the same for the
every-expert-on-every-token layer it replaces, and what the routed layer's skipped tiles saved.
Mixtral-8x7B's shape by default, random weights, synthetic tokens.
"""

from __future__ import annotations

import argparse
import json

import torch


def measure(members: int, tokens: int, hidden: int, inter: int, experts: int, top_k: int, iters: int = 20) -> dict:
    from ..ops import KernelOps
    from ..parallel.moe_a2a import ExpertAllToAll, default_cap

    dev = torch.device("cuda", torch.cuda.current_device())
    ops = KernelOps(dev)
    g = torch.Generator(device=dev).manual_seed(0)
    gu = [(torch.randn(2 * inter, hidden, generator=g, device=dev) * 0.02).bfloat16() for _ in range(experts)]
    dn = [(torch.randn(hidden, inter, generator=g, device=dev) * 0.02).bfloat16() for _ in range(experts)]
    x = torch.randn(members, tokens, hidden, generator=g, device=dev).bfloat16()
    logits = torch.randn(members * tokens, experts, generator=g, device=dev).bfloat16()
    ids, w = ops.moe_topk(logits, top_k)
    ids, w = ids.view(members, tokens, top_k).contiguous(), w.view(members, tokens, top_k).contiguous()
    a2a = ExpertAllToAll.emulated(dev, members, experts=experts, top_k=top_k, hidden=hidden, cap=default_cap(tokens))
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def routed():
        a2a(ops, x, ids, w, lambda e: gu[e], lambda e: dn[e])

    scale = ops.moe_route(logits, top_k, 0, experts)  # [E, members * tokens]
    flat = x.view(members * tokens, hidden)

    def replicated():  # every expert on every token, weights in the epilogue, experts summed in order
        acc = None
        for e in range(experts):
            acc = ops.linear(ops.silu_mul(ops.linear(flat, gu[e])), dn[e], scale=scale[e], pre=acc)

    def timed(fn) -> float:
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        total = 0.0
        for _ in range(iters):
            flush.fill_(1)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            fn()
            e.record()
            torch.cuda.synchronize()
            total += s.elapsed_time(e)
        return total / iters

    t_routed, t_rep = timed(routed), timed(replicated)
    status = [a2a.status(z) for z in range(members)]
    used = int(torch.unique(ids).numel())
    return {"metric": "routed mixture layer time (group emulated on one GPU)", "members": members,
            "tokens_per_member": tokens, "hidden": hidden, "inter": inter, "experts": experts, "top_k": top_k,
            "routed_ms": round(t_routed, 4), "every_expert_ms": round(t_rep, 4), "experts_chosen": used,
            "weight_bytes_per_expert": 3 * hidden * inter * 2, "status": status}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--members", type=int, default=4)
    ap.add_argument("--tokens", type=int, default=64)
    ap.add_argument("--hidden", type=int, default=4096)
    ap.add_argument("--inter", type=int, default=14336)
    ap.add_argument("--experts", type=int, default=8)
    ap.add_argument("--top-k", type=int, default=2)
    a = ap.parse_args()
    print(json.dumps(measure(a.members, a.tokens, a.hidden, a.inter, a.experts, a.top_k)))


if __name__ == "__main__":
    main()
