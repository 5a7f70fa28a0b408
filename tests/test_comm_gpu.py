"""Peer-memory collectives on 2+ GPUs (one process per GPU), against the rank-order fp32 oracle.

Skipped with fewer than two GPUs. The failure case injects nothing on the GPU: one rank simply does
not enter the call, the other's kernel names it late after the bound and leaves when the host
raises the abort word (a bounded wait; no trap, no fault).
"""

import os
import socket
import threading
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _tensor(rank: int, n: int, seed: int) -> torch.Tensor:
    g = torch.Generator(device="cpu").manual_seed(seed * 100 + rank)
    return torch.randn(n, generator=g).bfloat16()


def _worker(rank: int, world: int, port: int, results, nvls: bool = False):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    from datetime import timedelta

    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=timedelta(seconds=60))
    from everserve_b200.ops import KernelOps, ref
    from everserve_b200.parallel.fused import FusedTPCollective

    out = {}
    coll = FusedTPCollective(dev, nvls=nvls)
    try:
        # 1. fdar: bit-identical to the rank-order fp32 sum, every size including ragged tails
        ok = True
        for n in (8, 1000, 4096, 65536, 300001, 1 << 20):
            x = _tensor(rank, n, n).to(dev)
            y = coll.all_reduce(x.clone())
            expect = ref.member_sum([_tensor(r, n, n) for r in range(world)]).to(dev)
            ok &= bool(torch.equal(y, expect))
        out["fdar_exact"] = ok
        # 2. fused row-parallel GEMM + all-reduce vs unfused GEMM + member sum
        kops = KernelOps(dev)
        M, N, K = 37, 4096, 2048
        g = torch.Generator(device="cpu").manual_seed(7 + rank)
        xs = torch.randn(M, K, generator=g).bfloat16().to(dev)
        ws = (torch.randn(N, K, generator=g) / 64).bfloat16().to(dev)
        res = torch.randn(M, N, generator=torch.Generator().manual_seed(99)).bfloat16().to(dev)
        fused = coll.linear_allreduce(kops, xs, ws, residual=res)
        part = kops.linear(xs, ws)
        parts = [torch.empty_like(part) for _ in range(world)]
        dist.all_gather(parts, part)
        expect = (ref.member_sum(parts).float() + res.float())
        out["gemm_ar_close"] = bool(torch.allclose(fused.float(), expect, rtol=2e-2, atol=2e-2))
        # the fp32 oracle straight from the operands: every member's x_r . w_r^T, summed in rank order
        oracle = torch.zeros(M, N)
        for r in range(world):
            gr = torch.Generator(device="cpu").manual_seed(7 + r)
            xr = torch.randn(M, K, generator=gr).bfloat16()
            wr = (torch.randn(N, K, generator=gr) / 64).bfloat16()
            oracle += xr.float() @ wr.float().t()
        oracle += res.float().cpu()
        out["gemm_ar_oracle"] = bool(torch.allclose(fused.float().cpu(), oracle, rtol=2e-2, atol=3e-2))
        allf = [torch.empty_like(fused) for _ in range(world)]
        dist.all_gather(allf, fused)
        out["gemm_ar_same_on_ranks"] = all(torch.equal(allf[0], f) for f in allf)
        out["status"] = coll.status() + kops.check_status()
        # 2b. fused GEMMs of different K (so different cluster splits) back to back, as o_proj and
        # down_proj alternate in decode: the words of one must never be taken for the other's
        ok = True
        for it in range(6):
            for K2 in (512, 1792):
                g2 = torch.Generator(device="cpu").manual_seed(1000 + 10 * it + K2 + rank)
                x2 = torch.randn(64, K2, generator=g2).bfloat16().to(dev)
                w2 = (torch.randn(4096, K2, generator=torch.Generator().manual_seed(K2 + rank)) / 64).bfloat16().to(dev)
                f2 = coll.linear_allreduce(kops, x2, w2)
                p2 = kops.linear(x2, w2)
                ps2 = [torch.empty_like(p2) for _ in range(world)]
                dist.all_gather(ps2, p2)
                ok &= bool(torch.allclose(f2.float(), ref.member_sum(ps2).float(), rtol=2e-2, atol=2e-2))
        out["alternating_splits_close"] = ok
        out["status"] += coll.status() + kops.check_status()
        # 2c. the fused reduce-scatter and all-gather GEMMs (the sequence-parallel pair) against fp32
        ok_rs = ok_ag = True
        for it, M in enumerate((64, 37, 8)):
            K, N = 1024, 2048
            xs_r = [torch.randn(M, K, generator=torch.Generator().manual_seed(300 + 7 * it + r)).bfloat16()
                    for r in range(world)]
            ws_r = [(torch.randn(N, K, generator=torch.Generator().manual_seed(400 + 7 * it + r)) / 32).bfloat16()
                    for r in range(world)]
            per = -(-M // world)
            rs = coll.linear_reduce_scatter(kops, xs_r[rank].to(dev), ws_r[rank].to(dev))
            full = sum(x.float() @ wr.float().t() for x, wr in zip(xs_r, ws_r))
            lo, hi = min(M, rank * per), min(M, (rank + 1) * per)
            ok_rs &= bool(torch.allclose(rs[: hi - lo].float().cpu(), full[lo:hi], rtol=2e-2, atol=3e-2))
            # every member's own rows, gathered in member order, times this member's weight
            mine = [torch.randn(per, K, generator=torch.Generator().manual_seed(500 + 7 * it + r)).bfloat16()
                    for r in range(world)]
            ag = coll.gather_linear(kops, mine[rank].to(dev), ws_r[rank].to(dev))
            want = torch.cat(mine).float() @ ws_r[rank].float().t()
            ok_ag &= bool(torch.allclose(ag.float().cpu(), want, rtol=2e-2, atol=3e-2))
        out["rs_close"], out["ag_close"] = ok_rs, ok_ag
        out["status"] += coll.status() + kops.check_status()
        # 3. a member that never enters the call: named late, released by the abort word (P2P only:
        # no member of an NVLS group is ever left behind on this pool)
        torch.cuda.synchronize()
        dist.barrier()
        if nvls:
            results[rank] = out
            return
        coll.set_bound_ns(20_000_000)
        if rank == 0:
            x = torch.ones(4096, dtype=torch.bfloat16, device=dev)

            def raise_abort():
                time.sleep(0.3)
                coll.abort()

            t = threading.Thread(target=raise_abort)
            t.start()
            t0 = time.monotonic()
            coll.all_reduce(x)
            torch.cuda.synchronize()
            out["abort_s"] = time.monotonic() - t0
            t.join()
            out["late"] = coll.late_rows()
            out["abort_status"] = coll.status()
        dist.barrier()
        coll.resume()
        dist.barrier()
        # 4. the group works again after resume
        x = _tensor(rank, 4096, 5).to(dev)
        y = coll.all_reduce(x.clone())
        expect = ref.member_sum([_tensor(r, 4096, 5) for r in range(world)]).to(dev)
        out["after_resume"] = bool(torch.equal(y, expect))
    finally:
        torch.cuda.synchronize()
        dist.barrier()
        coll.close()
        dist.destroy_process_group()
    results[rank] = out


@pytest.mark.parametrize("nvls", [False, True])
def test_peer_collectives(nvls):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = min(torch.cuda.device_count(), 8)
    port = _free_port()
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    procs = [ctx.Process(target=_worker, args=(r, world, port, results, nvls)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = dict(results)
    for r in range(world):
        o = res[r]
        assert o["fdar_exact"], o
        assert o["gemm_ar_close"] and o["gemm_ar_same_on_ranks"] and o["gemm_ar_oracle"], o
        assert o["alternating_splits_close"], o
        if not nvls:
            assert o["rs_close"] and o["ag_close"], o
        assert o["status"] == 0, o
        if not nvls:
            assert o["after_resume"], o
    if nvls:
        return
    r0 = res[0]
    assert r0["abort_status"] == 2, r0
    assert 1 in r0["late"], r0
    assert r0["abort_s"] < 3.0, r0
