"""Small, self-ending launches of one kernel, sized for a profiler capture.

    python -m everserve_b200.perf.ncu_case --kernel gemm [--n 28672 --k 4096 --m 64]
    python -m everserve_b200.perf.ncu_case --kernel attn [--batch 64 --ctx 1024]
    python -m everserve_b200.perf.ncu_case --kernel prefill [--batch 16 --ctx 1024]
    python -m everserve_b200.perf.ncu_case --kernel gemm_ar|fdar [--n 4096 --k 512 --m 64]  (a one-member group)
    python -m everserve_b200.perf.ncu_case --kernel fp8 [--n 28672 --k 4096 --m 64]
    python -m everserve_b200.perf.ncu_case --kernel norm|rope|silu|argmax|kvgather

Each case allocates a few hundred MB at most (operands larger than the 126 MB L2 where the kernel
is bandwidth-bound, so DRAM counters mean something), runs ``--launches`` launches of the kernel
(3 by default: capture the last with ``-s 2 -c 1``) and exits. The shapes default to the
Llama-3-8B decode shapes at batch 64.
"""

from __future__ import annotations

import argparse
import math

import torch

from ..ops import KernelOps


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--kernel", required=True,
                    choices=["gemm", "attn", "prefill", "norm", "rope", "silu", "argmax", "kvgather", "gemm_ar", "fdar",
                             "fp8"])
    ap.add_argument("--m", type=int, default=64)
    ap.add_argument("--n", type=int, default=28672)
    ap.add_argument("--k", type=int, default=4096)
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--ctx", type=int, default=1024)
    ap.add_argument("--launches", type=int, default=3)
    ap.add_argument("--time", action="store_true", help="also print the CUDA-event time per launch")
    a = ap.parse_args()
    dev = torch.device("cuda", 0)
    ops = KernelOps(dev)
    coll = None
    C = ops.C
    g = torch.Generator(device=dev).manual_seed(0)
    if a.kernel == "gemm":
        w = torch.randn(a.n, a.k, device=dev, generator=g).bfloat16()
        x = torch.randn(a.m, a.k, device=dev, generator=g).bfloat16()
        ops.reserve_linear(a.m, [(a.n, a.k)])
        out = torch.empty(a.m, a.n, device=dev, dtype=torch.bfloat16)
        run = lambda: ops.linear(x, w, out=out)  # noqa: E731
    elif a.kernel == "attn":
        hq, hkv, d, bs = 32, 8, 128, 16
        mb = (a.ctx + bs - 1) // bs
        cache = torch.randn(a.batch * mb, 2, hkv, bs, d, device=dev, generator=g).bfloat16()
        bt = torch.arange(a.batch * mb, device=dev, dtype=torch.int32).view(a.batch, mb)
        cl = torch.full((a.batch,), a.ctx, device=dev, dtype=torch.int32)
        q = torch.randn(a.batch, hq, d, device=dev, generator=g).bfloat16()
        ops.reserve_attention(a.batch, hq, d, mb * bs)
        run = lambda: ops.decode_attention(q, cache, bt, cl, 1 / math.sqrt(d), mb * bs)  # noqa: E731
    elif a.kernel == "prefill":
        # `batch` prompts of `ctx` tokens prefilled at once (each sees its own causal history)
        from ..ops import prefill_tiles

        hq, hkv, d, bs = 32, 8, 128, 16
        mb = (a.ctx + bs - 1) // bs
        cache = torch.randn(a.batch * mb, 2, hkv, bs, d, device=dev, generator=g).bfloat16()
        bt = torch.arange(a.batch * mb, device=dev, dtype=torch.int32).view(a.batch, mb)
        cl = torch.full((a.batch,), a.ctx, device=dev, dtype=torch.int32)
        q = torch.randn(a.batch * a.ctx, hq, d, device=dev, generator=g).bfloat16()
        seq = [i for i in range(a.batch) for _ in range(a.ctx)]
        pos = [p for _ in range(a.batch) for p in range(a.ctx)]
        tiles = prefill_tiles(seq, pos, device=dev)
        qs, ps = torch.tensor(seq, device=dev), torch.tensor(pos, device=dev)
        run = lambda: ops.prefill_attention(q, cache, bt, cl, qs, ps, 1 / math.sqrt(d), tiles)  # noqa: E731
    elif a.kernel in ("gemm_ar", "fdar"):
        # the fused GEMM + all-reduce (or the all-reduce alone) in a group of one member on this GPU:
        # the kernel's full code path, its pushes going to this member's own buffer
        import os
        import socket

        import torch.distributed as dist

        from ..parallel.fused import FusedTPCollective

        sk = socket.socket()
        sk.bind(("127.0.0.1", 0))
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", str(sk.getsockname()[1]))
        sk.close()
        dist.init_process_group("gloo", rank=0, world_size=1)
        coll = FusedTPCollective(dev)
        if a.kernel == "gemm_ar":
            w = torch.randn(a.n, a.k, device=dev, generator=g).bfloat16()
            x = torch.randn(a.m, a.k, device=dev, generator=g).bfloat16()
            run = lambda: coll.linear_allreduce(ops, x, w)  # noqa: E731
        else:
            v = torch.randn(a.m * a.n, device=dev, generator=g).bfloat16()
            run = lambda: coll.all_reduce_into(v, v)  # noqa: E731
    elif a.kernel == "fp8":
        from ..ops import quantize_weight_fp8

        w8, ws = quantize_weight_fp8(torch.randn(a.n, a.k, device=dev, generator=g) / 64)
        x = torch.randn(a.m, a.k, device=dev, generator=g).bfloat16()
        run = lambda: ops.linear_fp8(x, w8, ws)  # noqa: E731
    elif a.kernel == "norm":
        x = torch.randn(a.batch * 64, 4096, device=dev, generator=g).bfloat16()
        r = torch.randn_like(x)
        wt = torch.randn(4096, device=dev, generator=g).bfloat16()
        run = lambda: ops.rmsnorm(x, wt, 1e-5, r)  # noqa: E731
    elif a.kernel == "silu":
        x = torch.randn(a.batch * 64, 2 * 14336, device=dev, generator=g).bfloat16()
        run = lambda: ops.silu_mul(x)  # noqa: E731
    elif a.kernel == "argmax":
        x = torch.randn(a.batch, 128256, device=dev, generator=g).bfloat16()
        run = lambda: ops.argmax(x)  # noqa: E731
    elif a.kernel == "rope":
        from ..ops import ref

        hq, hkv, d, bs = 32, 8, 128, 16
        n = a.batch
        qkv = torch.randn(n, (hq + 2 * hkv) * d, device=dev, generator=g).bfloat16()
        pos = torch.arange(n, device=dev) + a.ctx
        cs = ref.cos_sin_table(d, 8192, 5e5).to(dev)
        cache = torch.zeros(n, 2, hkv, bs, d, device=dev, dtype=torch.bfloat16)
        slots = torch.arange(n, device=dev) * bs
        run = lambda: ops.rope_kv_write(qkv, None, pos, cs, slots, cache, hq, hkv, bs)  # noqa: E731
    else:  # kvgather: one step's rows of 32 layers x 8 heads into a mapped host staging buffer
        from ..state.kvcopy import PagedKV

        layers, nb, bs, H, d = 32, 512, 16, 8, 128
        kv = PagedKV("heads_blocked", nb, bs, H, d)
        caches = [torch.randn(kv.shape(), device=dev, generator=g).bfloat16() for _ in range(layers)]
        ptrs = torch.tensor([c.data_ptr() for c in caches], dtype=torch.int64, device=dev)
        heads = torch.arange(H, device=dev)
        slots = torch.arange(a.batch, device=dev) * bs + 3
        cap = 64
        host = torch.empty(layers * H * cap * 2 * d, dtype=torch.bfloat16).pin_memory()
        dptr = host.data_ptr()  # pinned host memory is device-addressable under unified addressing
        run = lambda: C.kv_gather(ptrs, slots, heads, dptr, cap, d, bs, kv.strides(), 2)  # noqa: E731
    for _ in range(a.launches):
        run()
    torch.cuda.synchronize()
    print(f"{a.kernel}: {a.launches} launches done")
    if a.time:
        # CUDA-event time per launch after the launches above (warm); never read under a profiler
        flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
        ts = []
        for _ in range(10):
            flush.zero_()  # the operands leave L2 between launches
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            run()
            e.record()
            torch.cuda.synchronize()
            ts.append(s.elapsed_time(e) * 1e3)
        ts.sort()
        print(f"{a.kernel}: median {ts[len(ts) // 2]:.1f} us, min {ts[0]:.1f} us per launch (L2 flushed)")
    if coll is not None:
        # the collective's heartbeat thread and peer mappings go before the interpreter does
        torch.cuda.synchronize()
        coll.close()
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()
