"""Per-kernel timing at the decode shapes (CUDA events, warm, L2 flushed between launches).

    python -m everserve_b200.perf.kernels [--only gemm|attn] [--tp 1]

Reports achieved bandwidth against the algorithmic bytes of each launch (weights + activations for
a GEMM; K/V history + q/out for attention). Every launch is preceded by a write of a buffer larger
than L2 so weights come from HBM.
"""

from __future__ import annotations

import argparse
import json
import math

import torch

from ..ops import KernelOps, PackedWeight, pack_weight, ref


def _graph_ms(body, iters):
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(iters):
            body()
    g.replay()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    g.replay()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e)


def _time(fn, iters=20, flush=None):
    """Device time of one launch of fn: a graph of (flush, fn) x iters minus a graph of flushes."""
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    if flush is None:
        return _graph_ms(fn, iters) / iters

    def both():
        flush.zero_()
        fn()

    return (_graph_ms(both, iters) - _graph_ms(flush.zero_, iters)) / iters


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default=None)
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--ctx", type=int, default=1024)
    a = ap.parse_args()
    dev = torch.device("cuda", 0)
    k = KernelOps(dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    tp, M = a.tp, a.batch
    rows = []
    if a.only in (None, "gemm"):
        H, I, V = 4096, 14336, 128256
        shapes = {"qkv": (6144 // tp, H), "o": (H, 4096 // tp), "gate_up": (2 * I // tp, H), "down": (H, I // tp),
                  "lm_head": (V // tp, H)}
        for name, (N, K) in shapes.items():
            w = torch.randn(N, K, device=dev).bfloat16()
            x = torch.randn(M, K, device=dev).bfloat16()
            k.reserve_linear(M, [(N, K)])
            out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
            ms = _time(lambda: k.linear(x, w, out=out), flush=flush)
            cub = _time(lambda: torch.matmul(x, w.t(), out=out), flush=flush)
            byts = (N * K + M * K + M * N) * 2
            # the same launch with the weights still in L2 from the launch before (no flush): what
            # the GEMM would take if its weights were fetched into L2 while the kernel before ran
            hot = _time(lambda: k.linear(x, w, out=out))
            rows.append({"kernel": "gemm", "name": name, "M": M, "N": N, "K": K,
                         "us": round(ms * 1e3, 2), "gb_s": round(byts / ms / 1e6, 1),
                         "cublas_us": round(cub * 1e3, 2), "cublas_gb_s": round(byts / cub / 1e6, 1),
                         "l2_resident_us": round(hot * 1e3, 2)})
            # the same weights pre-packed into swizzled 16 KB blocks (one bulk copy per stage)
            wp = pack_weight(w)
            ref_out = k.linear(x, w).clone()
            pms = _time(lambda: k.linear(x, w, out=out, w_packed=wp), flush=flush)
            same = bool(torch.equal(k.linear(x, w, w_packed=wp), ref_out))
            rows.append({"kernel": "gemm_packed", "name": name, "M": M, "N": N, "K": K,
                         "us": round(pms * 1e3, 2), "gb_s": round(byts / pms / 1e6, 1), "equal_to_tiled": same})
            del wp
            if name == "gate_up" and M <= 64:
                # the same weights with SiLU-mul in the GEMM epilogue (rows interleaved by 64)
                sms = _time(lambda: k.linear_silu(x, w), flush=flush)
                byts_s = (N * K + M * K + M * N // 2) * 2
                rows.append({"kernel": "gemm_silu", "name": name, "M": M, "N": N, "K": K,
                             "us": round(sms * 1e3, 2), "gb_s": round(byts_s / sms / 1e6, 1)})
                # and pre-packed, as the decode step runs it
                pw = PackedWeight(w)
                pss = _time(lambda: k.linear_silu(x, pw), flush=flush)
                rows.append({"kernel": "gemm_silu_packed", "name": name, "M": M, "N": N, "K": K,
                             "us": round(pss * 1e3, 2), "gb_s": round(byts_s / pss / 1e6, 1)})
                del pw
    if a.only in (None, "attn"):
        hq, hkv, d, bs = 32 // tp, max(1, 8 // tp), 128, 16
        B, ctx = M, a.ctx
        mb = (ctx + 64 + bs - 1) // bs
        cache = torch.randn(B * mb, 2, hkv, bs, d, device=dev).bfloat16()
        bt = torch.arange(B * mb, device=dev, dtype=torch.int32).view(B, mb)
        cl = torch.full((B,), ctx, device=dev, dtype=torch.int32)
        q = torch.randn(B, hq, d, device=dev).bfloat16()
        for part in (256, 512):
            for stages in (2, 3, 4):
                k.PART_TOKENS, k.ATTN_STAGES = part, stages
                k.reserve_attention(B, hq, d, mb * bs)
                ms = _time(lambda: k.decode_attention(q, cache, bt, cl, 1 / math.sqrt(d), mb * bs), flush=flush)
                byts = B * ctx * 2 * hkv * d * 2
                rows.append({"kernel": "paged_decode", "B": B, "ctx": ctx, "hq": hq, "hkv": hkv, "part": part,
                             "stages": stages, "us": round(ms * 1e3, 2), "gb_s": round(byts / ms / 1e6, 1)})
        _ = ref
    if a.only in (None, "sample"):
        # seeded top-k / top-p sampling of the batch's rows over the 8B vocabulary: the kernel
        # against the host sampler (tensor ops: sort, softmax, cumsum, scatter)
        from ..engine.sampling import SamplingBatch, sample

        V = 128256
        logits = (torch.randn(M, V, device=dev) * 2.5).bfloat16()
        pos = torch.arange(M, device=dev, dtype=torch.int64)
        for name, tk, tp in (("temperature", 0, 1.0), ("top_k50", 50, 1.0), ("top_p0.9", 0, 0.9),
                             ("top_k50_p0.9", 50, 0.9)):
            sb = SamplingBatch(temperature=torch.full((M,), 0.8, device=dev),
                               top_k=torch.full((M,), tk, dtype=torch.int64, device=dev),
                               top_p=torch.full((M,), tp, device=dev), seed=torch.arange(M, device=dev) + 7)
            ms = _time(lambda: k.sample(logits, pos, sb), flush=flush)
            hms = _time(lambda: sample(logits, pos, sb), iters=5)
            rows.append({"kernel": "sample", "name": name, "B": M, "V": V, "us": round(ms * 1e3, 2),
                         "host_sampler_us": round(hms * 1e3, 2)})
    for r in rows:
        print(json.dumps(r))


if __name__ == "__main__":
    main()
