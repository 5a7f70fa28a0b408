"""Sequence parallelism on the CPU tier (two gloo ranks): the token-sliced forward (norms on each
rank's slice, reduce-scatter after the row-parallel projections, all-gather before the column-parallel
ones) gives the tensor-parallel forward's logits, in prefill and in decode, with a token count that
does not divide by the ranks (padding rows)."""

import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from everserve_b200.models.config import TINY_LLAMA
from everserve_b200.models.llama import DecoderLM, StepInput, TPGroup
from everserve_b200.parallel.nccl import GroupCollective


def _port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _inputs(T: int, bs: int = 16):
    ids = torch.arange(T) * 37 % TINY_LLAMA.vocab
    pos = torch.arange(T)
    bt = torch.arange(8, dtype=torch.int32)[None]
    return StepInput(ids=ids, positions=pos, slots=pos.clone(), block_tables=bt,
                     ctx_lens=torch.tensor([T], dtype=torch.int32), q_seq=torch.zeros(T, dtype=torch.int64),
                     logits_idx=torch.tensor([T - 1]), is_decode=False)


def _decode_inputs(B: int, ctx: int):
    """B sequences of one new token each at position ctx - 1 (histories written by `_fill`)."""
    bt = torch.stack([torch.arange(8, dtype=torch.int32) + 8 * b for b in range(B)])
    pos = torch.full((B,), ctx - 1)
    return StepInput(ids=torch.arange(B) + 3, positions=pos, slots=bt[:, (ctx - 1) // 16].long() * 16 + (ctx - 1) % 16,
                     block_tables=bt, ctx_lens=torch.full((B,), ctx, dtype=torch.int32), q_seq=torch.arange(B),
                     logits_idx=torch.arange(B), is_decode=True)


def _worker(rank: int, port: int, out):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=2)
    try:
        res = {}
        for sp in (False, True):
            tp = TPGroup(rank, 2, GroupCollective(None))
            m = DecoderLM(TINY_LLAMA, "cpu", torch.float32, seed=1, tp=tp, sequence_parallel=sp)
            g = torch.Generator().manual_seed(7)
            caches = [torch.randn(m.kv_cache_shape(32, 16), generator=g) * 0.1 for _ in range(TINY_LLAMA.layers)]
            pre = m.logits(_inputs(13), [c.clone() for c in caches])  # 13 tokens: 7 + 6 over two ranks
            dec = m.logits(_decode_inputs(3, 20), [c.clone() for c in caches])  # 3 rows: 2 + 1 (+ padding)
            res[sp] = (pre, dec)
        out[rank] = {k: (v[0].numpy(), v[1].numpy()) for k, v in res.items()}
    finally:
        dist.destroy_process_group()


def test_sequence_parallel_matches_tensor_parallel():
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, port, out)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=180)
    assert all(p.exitcode == 0 for p in ps), [p.exitcode for p in ps]
    for r in range(2):
        (pre_tp, dec_tp), (pre_sp, dec_sp) = out[r][False], out[r][True]
        assert abs(pre_tp - pre_sp).max() < 1e-4 and abs(dec_tp - dec_sp).max() < 1e-4
        assert (pre_tp.argmax(-1) == pre_sp.argmax(-1)).all() and (dec_tp.argmax(-1) == dec_sp.argmax(-1)).all()
