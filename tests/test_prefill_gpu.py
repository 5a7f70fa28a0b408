"""The tcgen05 paged prefill attention kernel against the fp32 PyTorch oracle of the same op.

Ragged batches: sequences of different lengths, chunks that start after earlier chunks (the history
comes from the cache), lengths that are not multiples of the 128-row tile or the block size, block
tables in shuffled order, GQA group sizes 1 to 8, head sizes 64 and 128, block sizes 16 and 32.
"""

import math

import pytest
import torch

from everserve_b200.ops import KernelOps, prefill_tiles, ref

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def kops():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return KernelOps("cuda:0")


def _case(seed, chunks, hq, hkv, d, bs):
    """chunks: (history, new rows) per sequence. Returns q, cache, tables, ctx, q_seq, q_pos."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    max_ctx = max(h + n for h, n in chunks)
    mb = (max_ctx + bs - 1) // bs
    nb = len(chunks) * mb + 3
    cache = torch.randn(nb, 2, hkv, bs, d, device="cuda", generator=g).bfloat16()
    bt = torch.randperm(nb, device="cuda", generator=g)[: len(chunks) * mb].view(len(chunks), mb).int().contiguous()
    T = sum(n for _, n in chunks)
    q = torch.randn(T, hq, d, device="cuda", generator=g).bfloat16()
    q_seq, q_pos = [], []
    for i, (h, n) in enumerate(chunks):
        q_seq += [i] * n
        q_pos += list(range(h, h + n))
    ctx = torch.tensor([h + n for h, n in chunks], dtype=torch.int32, device="cuda")
    return q, cache, bt, ctx, torch.tensor(q_seq, device="cuda"), torch.tensor(q_pos, device="cuda")


def _oracle(q, cache, bt, ctx, q_seq, q_pos, scale):
    return ref.paged_attention(q.float(), cache.float(), bt, ctx, q_seq, q_pos, scale)


@pytest.mark.parametrize("hq,hkv,d,bs", [(32, 8, 128, 16), (8, 8, 128, 16), (14, 2, 64, 16), (16, 2, 128, 32),
                                         (8, 1, 64, 32)])
def test_prefill_matches_oracle(kops, hq, hkv, d, bs):
    chunks = [(0, 1), (0, 127), (0, 128), (0, 129), (0, 300), (17, 5), (250, 260), (1000, 64), (3, 1)]
    q, cache, bt, ctx, q_seq, q_pos = _case(1, chunks, hq, hkv, d, bs)
    scale = 1.0 / math.sqrt(d)
    out = kops.prefill_attention(q, cache, bt, ctx, q_seq, q_pos, scale,
                                 prefill_tiles(q_seq.tolist(), q_pos.tolist(), device="cuda"))
    torch.cuda.synchronize()
    assert kops.check_status() == 0
    want = _oracle(q, cache, bt, ctx, q_seq, q_pos, scale)
    torch.testing.assert_close(out.float(), want.float(), rtol=2e-2, atol=2e-2)


def test_prefill_rows_independent_of_batch(kops):
    """A sequence's rows come out the same whatever else shares the launch (batch invariance)."""
    chunks = [(0, 200), (64, 100)]
    q, cache, bt, ctx, q_seq, q_pos = _case(2, chunks, 32, 8, 128, 16)
    scale = 1.0 / math.sqrt(128)
    both = kops.prefill_attention(q, cache, bt, ctx, q_seq, q_pos, scale)
    alone = kops.prefill_attention(q[:200].contiguous(), cache, bt[:1], ctx[:1], q_seq[:200], q_pos[:200], scale)
    torch.cuda.synchronize()
    assert torch.equal(both[:200], alone)


def test_prefill_long_context(kops):
    """Every KV tile of a 4096-position history passes through the two-stage ring."""
    chunks = [(3968, 128), (0, 2048)]
    q, cache, bt, ctx, q_seq, q_pos = _case(3, chunks, 32, 8, 128, 16)
    scale = 1.0 / math.sqrt(128)
    out = kops.prefill_attention(q, cache, bt, ctx, q_seq, q_pos, scale)
    torch.cuda.synchronize()
    assert kops.check_status() == 0
    want = _oracle(q, cache, bt, ctx, q_seq, q_pos, scale)
    torch.testing.assert_close(out.float(), want.float(), rtol=2e-2, atol=2e-2)
