"""Sequence parallelism on 2+ GPUs: the decoder's token-sliced forward on the fused reduce-scatter
and all-gather GEMMs gives the same tokens as the tensor-parallel forward on the fused all-reduce
GEMM, in prefill and decode, and leaves no status word set."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank: int, world: int, port: int, out):
    from datetime import timedelta

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world, device_id=dev,
                            timeout=timedelta(seconds=60))
    from everserve_b200.engine import Engine, EngineConfig, LocalExecutor
    from everserve_b200.models.config import SMALL_LLAMA
    from everserve_b200.parallel.fused import FusedTPCollective

    coll = FusedTPCollective(dev)
    res = {}
    try:
        for sp in (False, True):
            cfg = EngineConfig(SMALL_LLAMA, device=str(dev), max_batch=16, max_model_len=256, num_blocks=128,
                               tensor_parallel=world, use_cuda_graphs=False, sequence_parallel=sp)
            eng = Engine(cfg, executor=LocalExecutor(cfg, rank=rank, collective=coll))
            prompts = [list(range(5 + i, 40 + 3 * i)) for i in range(5)]
            res[sp] = eng.generate(prompts, max_tokens=8)
            res[f"status{sp}"] = eng.executor.worker.model.ops.check_status() + coll.status()
            eng.executor.worker.runner.release_graphs()
        out[rank] = res
    finally:
        torch.cuda.synchronize()
        dist.barrier()
        coll.close()
        dist.destroy_process_group()


def test_sequence_parallel_tokens_match():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, out)) for r in range(world)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=300)
    for p in ps:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in ps), [p.exitcode for p in ps]
    for r in range(world):
        o = out[r]
        assert o[True] == o[False], (o[True], o[False])
        assert o["statusFalse"] == 0 and o["statusTrue"] == 0
