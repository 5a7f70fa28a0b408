"""The expert-parallel all-to-all kernels against the dense fp32 oracle.

On one GPU, ``ExpertAllToAll.emulated`` plays every member in one launch per step (local buffers);
with two or more GPUs, one process per GPU runs the real thing over peer-mapped VMM buffers. The
failure case injects nothing on the GPU: the owners' ready flags are never raised and the host's
abort word ends the combine's bounded wait with the aborted status.
"""

import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _weights(E, H, I, device, seed=0):
    g = torch.Generator().manual_seed(seed)
    gu = [(torch.randn(2 * I, H, generator=g) * 0.05).bfloat16().to(device) for _ in range(E)]
    dn = [(torch.randn(H, I, generator=g) * 0.05).bfloat16().to(device) for _ in range(E)]
    return gu, dn


def _oracle_expert(gu, dn):
    def f(e, rows):
        a = rows.float() @ gu[e].float().t()
        i = a.shape[1] // 2
        return (torch.nn.functional.silu(a[:, :i]) * a[:, i:]) @ dn[e].float().t()
    return f


def _close(got, want):
    err = (got.float() - want.float()).norm() / want.float().norm().clamp_min(1e-6)
    return float(err)


def _inputs(W, T, H, E, k, device, seed, avoid=None):
    from everserve_b200.ops import KernelOps

    ops = KernelOps(device)
    g = torch.Generator().manual_seed(seed)
    xs = torch.randn(W, T, H, generator=g).bfloat16().to(device)
    logits = torch.randn(W, T, E, generator=g)
    if avoid is not None:
        logits[..., avoid] = -30.0
    logits = logits.bfloat16().to(device)
    routed = [ops.moe_topk(logits[z], k) for z in range(W)]
    ids = torch.stack([r[0] for r in routed]).contiguous()
    ws = torch.stack([r[1] for r in routed]).contiguous()
    return ops, xs, logits, ids, ws


@pytest.mark.parametrize("W", [2, 4])
def test_emulated_group_matches_the_dense_oracle(W):
    from everserve_b200.ops import ref
    from everserve_b200.parallel.moe_a2a import ExpertAllToAll, default_cap

    dev = torch.device("cuda", 0)
    E, k, H, I, T = 8, 2, 256, 128, 37
    gu, dn = _weights(E, H, I, dev)
    a2a = ExpertAllToAll.emulated(dev, W, experts=E, top_k=k, hidden=H, cap=default_cap(T))
    for call, seed in enumerate((1, 2, 3)):  # the call counter advances between calls
        avoid = 5 if call == 2 else None
        ops, xs, logits, ids, ws = _inputs(W, T, H, E, k, dev, seed, avoid)
        rid, rw = ref.moe_topk(logits[0].cpu(), k)
        assert torch.equal(ids[0].cpu(), rid) and torch.allclose(ws[0].cpu(), rw, atol=1e-5)
        if avoid is not None:  # no token chose expert 5: its tiles are skipped and its outputs untouched
            z5, l5 = avoid // a2a.el, avoid % a2a.el
            a2a.expert_out(l5, z5).fill_(7.0)
        place = a2a.dispatch(xs, ids)
        a2a.run_experts(ops, lambda e: gu[e], lambda e: dn[e])
        a2a.ready()
        out = a2a.combine(ids, ws, place, ops.num_sms)
        torch.cuda.synchronize()
        want = ref.moe_a2a([x.float() for x in xs], list(ids), list(ws), _oracle_expert(gu, dn))
        for z in range(W):
            assert torch.equal(place[z].cpu(), ref.expert_places(ids[z].cpu(), E)), (call, z)
            assert _close(out[z], want[z]) < 2e-2, (call, z)
            assert a2a.status(z) == 0
        for d in range(W):  # every owner counted what each sender sent its experts
            for l in range(a2a.el):
                e = d * a2a.el + l
                sent = torch.tensor([int((ids[p] == e).sum()) for p in range(W)], dtype=torch.int32)
                assert torch.equal(a2a.counts(l, d).cpu(), sent), (d, l)
        if avoid is not None:
            assert bool((a2a.expert_out(l5, z5) == 7.0).all())


def test_grouped_gemm_skips_tiles_without_rows():
    from everserve_b200.ops import KernelOps

    dev = torch.device("cuda", 0)
    ops = KernelOps(dev)
    cap, segs, K, N = 64, 4, 256, 384
    g = torch.Generator().manual_seed(4)
    x = torch.randn(cap * segs, K, generator=g).bfloat16().to(dev)
    w = (torch.randn(N, K, generator=g) * 0.05).bfloat16().to(dev)
    valid = torch.tensor([3, 0, 64, 10], dtype=torch.int32, device=dev)
    out = torch.full((cap * segs, N), 7.0, dtype=torch.bfloat16, device=dev)
    ops.linear(x, w, out=out, valid=valid, valid_cap=cap)
    want = x.float() @ w.float().t()
    for s, n in enumerate(valid.tolist()):
        rows = slice(s * cap, s * cap + n)
        assert _close(out[rows], want[rows]) < 1e-2 if n else True
    none = torch.zeros(segs, dtype=torch.int32, device=dev)
    out2 = torch.full((cap * segs, N), 7.0, dtype=torch.bfloat16, device=dev)
    ops.linear(x, w, out=out2, valid=none, valid_cap=cap)
    torch.cuda.synchronize()
    assert bool((out2 == 7.0).all())  # no tile held a row: nothing ran
    assert ops.check_status() == 0


def test_abort_ends_the_combine_wait_with_a_status():
    from everserve_b200.ops import ref
    from everserve_b200.parallel.moe_a2a import CTRL_BYTES, ExpertAllToAll, default_cap

    dev = torch.device("cuda", 0)
    W, E, k, H, I, T = 2, 4, 2, 128, 64, 9
    gu, dn = _weights(E, H, I, dev)
    a2a = ExpertAllToAll.emulated(dev, W, experts=E, top_k=k, hidden=H, cap=default_cap(T))
    ops, xs, _, ids, ws = _inputs(W, T, H, E, k, dev, 5)
    place = a2a.dispatch(xs, ids)
    a2a.run_experts(ops, lambda e: gu[e], lambda e: dn[e])
    ctrl = a2a._keep[1].view(torch.int32)
    for z in range(W):
        ctrl[z * CTRL_BYTES // 4] = 1  # the host's abort word; no ready flag will come
    t0 = time.monotonic()
    a2a.combine(ids, ws, place, ops.num_sms)
    torch.cuda.synchronize()
    assert time.monotonic() - t0 < 3.0
    assert [a2a.status(z) for z in range(W)] == [2] * W
    ctrl.zero_()
    a2a.resume()
    out = a2a(ops, xs, ids, ws, lambda e: gu[e], lambda e: dn[e])
    torch.cuda.synchronize()
    want = ref.moe_a2a([x.float() for x in xs], list(ids), list(ws), _oracle_expert(gu, dn))
    assert all(_close(out[z], want[z]) < 2e-2 for z in range(W))


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    from datetime import timedelta

    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=timedelta(seconds=60))
    from everserve_b200.ops import ref
    from everserve_b200.parallel.fused import FusedTPCollective
    from everserve_b200.parallel.moe_a2a import ExpertAllToAll, default_cap

    out = {}
    coll = FusedTPCollective(dev)
    E, k, H, I, T = 8, 2, 512, 256, 50
    gu, dn = _weights(E, H, I, dev)
    a2a = ExpertAllToAll.over(coll, experts=E, top_k=k, hidden=H, cap=default_cap(T))
    try:
        errs = []
        for seed in (11, 12):
            ops, xs, _, ids, ws = _inputs(1, T, H, E, k, dev, seed * 10 + rank)
            got = a2a(ops, xs, ids, ws, lambda e: gu[e], lambda e: dn[e])
            torch.cuda.synchronize()
            want = ref.moe_a2a([xs[0].float()], [ids[0]], [ws[0]], _oracle_expert(gu, dn))[0]
            errs.append(_close(got[0], want))
        out["err"] = max(errs)
        # a mixture layer of the model: routed tokens agree with every-expert-on-every-token
        if E % world == 0:
            import dataclasses

            from everserve_b200.models.config import TINY_MIXTRAL
            from everserve_b200.models.llama import DecoderLM, TPGroup

            cfg = dataclasses.replace(TINY_MIXTRAL, num_experts=8)
            model = DecoderLM(cfg, dev, torch.bfloat16, 0, TPGroup(rank, world, coll))
            g = torch.Generator().manual_seed(99)
            layer_errs, routed_a2a = [], None
            for T in (1, 5, 70):  # fewer tokens than ranks, uneven slices, several per rank
                h = torch.randn(T, cfg.hidden, generator=g).bfloat16().to(dev)
                model.a2a = None
                dense = model._moe(h, "l0.")
                if routed_a2a is None:
                    assert model.enable_routed_experts(128)
                    routed_a2a = model.a2a
                model.a2a = routed_a2a
                model.ROUTED_MIN_TOKENS = 1  # route every step size under test
                routed = model._moe(h, "l0.")
                model.ROUTED_MIN_TOKENS = 1 << 30
                torch.cuda.synchronize()
                layer_errs.append(_close(routed, dense))
            out["layer_err"] = max(layer_errs)
        out["status"] = coll.status()
    finally:
        dist.barrier()
        a2a.close()
        coll.close()
        dist.destroy_process_group()
    results[rank] = out


def test_all_to_all_across_gpus():
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs two GPUs")
    world = 8 if n >= 8 else (4 if n >= 4 else 2)
    port = _free_port()
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    procs = [ctx.Process(target=_worker, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    for r in range(world):
        assert results[r]["err"] < 2e-2 and results[r]["status"] == 0, (r, results[r])
        assert results[r].get("layer_err", 0.0) < 3e-2, (r, results[r])


def test_routed_experts_on_one_gpu():
    """On one GPU a prefill-size mixture step routes its tokens within the GPU (a group of one)
    and agrees with running every expert on every token; a decode-size step keeps the latter."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from everserve_b200.models.config import get_config
    from everserve_b200.models.llama import DecoderLM

    dev = torch.device("cuda", 0)
    cfg = get_config("tiny-mixtral")
    model = DecoderLM(cfg, dev, torch.bfloat16, 0)
    g = torch.Generator().manual_seed(3)
    for T in (600, 1037):
        h = torch.randn(T, cfg.hidden, generator=g).bfloat16().to(dev)
        model.a2a = None
        dense = model._moe(h, "l0.")
        assert model.enable_routed_experts(2048)
        routed = model._moe(h, "l0.")
        torch.cuda.synchronize()
        assert _close(routed, dense) < 3e-2
        assert model.a2a.status() == 0
    small = torch.randn(64, cfg.hidden, generator=g).bfloat16().to(dev)
    a2a, model.a2a = model.a2a, None
    ref_small = model._moe(small, "l0.")
    model.a2a = a2a
    assert torch.equal(model._moe(small, "l0."), ref_small)  # below the threshold: the same path

