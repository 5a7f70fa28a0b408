"""The sampling kernel against a float64 oracle of the same draw (and the host sampler).

Rows mix greedy, temperature-only, top-k, top-p and top-k + top-p, over bf16 logits of the 8B
model's vocabulary (many tied values, so the index order among ties is exercised). The oracle
sorts (stable), applies the filters with float64 masses and takes the Gumbel-max of the same
counter-based uniforms. Rows whose top-p cut-off lies within 1e-6 of a running mass are left out
of the top-p comparison (a rounding there may move the cut-off by one token in either direction).
"""

import pytest
import torch

from everserve_b200.engine.sampling import SamplingBatch, sample, uniforms

pytestmark = pytest.mark.gpu

V = 128256


def _oracle(logits, positions, sb):
    x = logits.double()
    B, Vv = x.shape
    temp = sb.temperature.double().clamp(min=1e-6)
    # the kernel divides in float32, as the host sampler does
    z32 = logits.float() / sb.temperature.float().clamp(min=1e-6)[:, None]
    z = z32.double()
    sz, order = torch.sort(z32, dim=1, descending=True, stable=True)
    sz = sz.double()
    rank = torch.arange(Vv, device=x.device)[None, :]
    k = torch.where(sb.top_k > 0, sb.top_k.clamp(max=Vv), torch.full_like(sb.top_k, Vv))
    keep = rank < k[:, None]
    p = torch.softmax(sz, dim=1)
    before = torch.cumsum(p, dim=1) - p
    tp = sb.top_p.double()[:, None]
    keep &= (before < tp) | (rank == 0) | (tp >= 1)
    active = ((tp > 0) & (tp < 1))[:, 0]
    margin = torch.where(active, (before - tp).abs().min(dim=1).values,
                         torch.full((B,), 1.0, dtype=torch.float64, device=x.device))
    kept = torch.zeros_like(keep).scatter(1, order, keep)
    g = -torch.log(-torch.log(uniforms(sb.seed, positions, Vv)))
    s = torch.where(kept, z + g, torch.full_like(g, float("-inf")))
    drawn = s.argmax(dim=1)
    greedy = logits.float().argmax(dim=1)
    _ = temp
    return torch.where(sb.temperature > 0, drawn, greedy), margin


def _batch(B, dev, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    logits = (torch.randn(B, V, generator=g) * 2.5).bfloat16().to(dev)
    temp = torch.tensor([0.0, 1.0, 0.7, 1.3] * (B // 4), dtype=torch.float32)
    top_k = torch.tensor([0, 0, 50, 1, 0, 2000, 0, 40] * (B // 8), dtype=torch.int64)
    top_p = torch.tensor([1.0, 0.9, 1.0, 0.5, 0.95, 1.0, 0.3, 0.8] * (B // 8), dtype=torch.float32)
    seeds = torch.randint(0, 1 << 62, (B,), generator=g, dtype=torch.int64)
    pos = torch.randint(0, 4096, (B,), generator=g, dtype=torch.int64)
    sb = SamplingBatch(temperature=temp.to(dev), top_k=top_k.to(dev), top_p=top_p.to(dev), seed=seeds.to(dev))
    return logits, pos.to(dev), sb


@pytest.fixture(scope="module")
def kops():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from everserve_b200.ops import KernelOps

    return KernelOps(torch.device("cuda", 0))


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_kernel_matches_the_float64_oracle(kops, seed):
    logits, pos, sb = _batch(64, torch.device("cuda", 0), seed)
    got = kops.sample(logits, pos, sb)
    want, margin = _oracle(logits, pos, sb)
    clear = margin > 1e-6
    assert int(clear.sum()) >= 56
    assert torch.equal(got[clear], want[clear]), (got[clear] != want[clear]).nonzero()
    # deterministic: the same inputs draw the same tokens
    assert torch.equal(kops.sample(logits, pos, sb), got)
    # the host sampler agrees wherever the cut-off is clear of roundings
    host = sample(logits, pos, sb)
    assert torch.equal(host[clear], got[clear])


def test_strided_rows_and_fp32_logits(kops):
    dev = torch.device("cuda", 0)
    logits, pos, sb = _batch(16, dev, 5)
    padded = torch.zeros(16, V + 64, dtype=torch.bfloat16, device=dev)
    padded[:, :V] = logits
    a = kops.sample(padded[:, :V], pos, sb)
    b = kops.sample(logits, pos, sb)
    c = kops.sample(logits.float(), pos, sb)
    assert torch.equal(a, b) and torch.equal(b, c)


def test_filters_keep_what_they_promise(kops):
    """top_k = 1 is greedy; top_p <= 0 keeps the top token; ties go to the lowest index."""
    dev = torch.device("cuda", 0)
    B = 8
    logits = torch.zeros(B, V, dtype=torch.bfloat16, device=dev)
    logits[:, 1000] = 5.0
    logits[:, 77] = 5.0  # a tie with a lower index
    sb = SamplingBatch(temperature=torch.full((B,), 1.0, device=dev),
                       top_k=torch.tensor([1, 1, 0, 0, 2, 2, 0, 3], device=dev),
                       top_p=torch.tensor([1.0, 0.5, 0.0, -1.0, 1.0, 1.0, 1e-9, 1.0], device=dev),
                       seed=torch.arange(B, device=dev))
    pos = torch.zeros(B, dtype=torch.int64, device=dev)
    got = kops.sample(logits, pos, sb).tolist()
    assert got[0] == got[1] == got[2] == got[3] == got[6] == 77
    assert got[4] in (77, 1000) and got[5] in (77, 1000)
    # top_k 3 keeps the two peaks and the first zero-logit token (index 0)
    assert got[7] in (0, 77, 1000)
