"""Numerics of the sm_100a kernels against fp32 PyTorch references of the same ops."""

import math

import pytest
import torch

from everserve_b200 import _ext
from everserve_b200.ops import KernelOps, ref

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def kops():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return KernelOps("cuda:0")


def close(a, b, rtol=2e-2, atol=2e-2):
    torch.testing.assert_close(a.float(), b.float(), rtol=rtol, atol=atol)


def test_extension_is_native():
    C = _ext.load()
    assert C.__file__.endswith(".so")


@pytest.mark.parametrize("hidden", [256, 896, 4096, 8192])
@pytest.mark.parametrize("rows", [1, 7, 64])
def test_rmsnorm(kops, hidden, rows):
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(rows, hidden, device="cuda", generator=g).bfloat16()
    w = (1 + 0.1 * torch.randn(hidden, device="cuda", generator=g)).bfloat16()
    y = kops.rmsnorm(x, w, 1e-5)
    close(y, ref.rmsnorm(x.float(), w.float(), 1e-5))
    r = torch.randn(rows, hidden, device="cuda", generator=g).bfloat16()
    r_ref = r.clone()
    y2 = kops.rmsnorm(x, w, 1e-5, residual=r)
    expect_r = (x.float() + r_ref.float()).bfloat16()
    assert torch.equal(r, expect_r)
    close(y2, ref.rmsnorm(expect_r.float(), w.float(), 1e-5))


@pytest.mark.parametrize("hq,hkv,d,bias", [(32, 8, 128, False), (14, 2, 64, True), (4, 1, 128, False)])
def test_rope_kv_write(kops, hq, hkv, d, bias):
    T, bs, nb = 37, 16, 8
    g = torch.Generator(device="cuda").manual_seed(1)
    qkv = torch.randn(T, (hq + 2 * hkv) * d, device="cuda", generator=g).bfloat16()
    b = torch.randn((hq + 2 * hkv) * d, device="cuda", generator=g).bfloat16() if bias else None
    cs = ref.cos_sin_table(d, 4096, 5e5).cuda()
    pos = torch.randint(0, 4000, (T,), device="cuda", generator=g)
    slots = torch.randperm(nb * bs, device="cuda", generator=g)[:T]
    slots[3] = -1
    cache = torch.zeros(nb, 2, hkv, bs, d, device="cuda", dtype=torch.bfloat16)
    cache_ref = cache.clone().float()
    q = kops.rope_kv_write(qkv, b, pos, cs, slots, cache, hq, hkv, bs)
    q_ref = ref.rope_kv_write(qkv.float(), None if b is None else b.float(), pos, cs, slots, cache_ref, hq, hkv, bs)
    close(q, q_ref)
    close(cache, cache_ref)


def test_silu_mul_embed_argmax(kops):
    g = torch.Generator(device="cuda").manual_seed(2)
    gu = torch.randn(19, 2 * 1024, device="cuda", generator=g).bfloat16()
    close(kops.silu_mul(gu), ref.silu_mul(gu.float()))
    table = torch.randn(1000, 256, device="cuda", generator=g).bfloat16()
    ids = torch.randint(0, 1000, (33,), device="cuda", generator=g)
    assert torch.equal(kops.embed(ids, table), table[ids])
    logits = torch.randn(9, 128256, device="cuda", generator=g).bfloat16()
    logits[2, 5] = 100.0
    logits[2, 7] = 100.0  # tie: the lower index wins
    am = kops.argmax(logits)
    assert torch.equal(am, torch.argmax(logits.float(), dim=-1))
    assert am[2].item() == 5
    odd = torch.randn(3, 1001, device="cuda", generator=g).bfloat16()
    assert torch.equal(kops.argmax(odd), torch.argmax(odd.float(), dim=-1))


GEMM_SHAPES = [
    (1, 128, 64), (7, 200, 256), (16, 4096, 4096), (33, 6144, 4096), (64, 4096, 14336),
    (64, 28672, 4096), (100, 512, 1024), (256, 1024, 512), (300, 768, 4096), (1000, 4096, 896),
    (64, 4096, 512), (64, 1000, 1792), (5, 384, 4104),
    # tensor-parallel-8 shapes of the 8B model: qkv (6 tiles), o, gate_up, down, lm_head shard
    (64, 768, 4096), (64, 4096, 512), (64, 3584, 4096), (64, 4096, 1792), (64, 16032, 4096),
]


@pytest.mark.parametrize("M,N,K", GEMM_SHAPES)
def test_gemm(kops, M, N, K):
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N + K)
    x = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    w = (torch.randn(N, K, device="cuda", generator=g) / math.sqrt(K)).bfloat16()
    y = kops.linear(x, w)
    expect = x.float() @ w.float().t()
    close(y, expect, rtol=2e-2, atol=2e-2)
    assert kops.check_status() == 0


def test_gemm_residual_and_repeat(kops):
    g = torch.Generator(device="cuda").manual_seed(3)
    M, N, K = 48, 4096, 4096
    x = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    w = (torch.randn(N, K, device="cuda", generator=g) / 64).bfloat16()
    r = torch.randn(M, N, device="cuda", generator=g).bfloat16()
    y = kops.linear(x, w, residual=r)
    close(y, x.float() @ w.float().t() + r.float())
    # the same product twice (stream-K fixup in CTA order) gives the same bits, across shapes
    # that change how the work splits between CTAs
    a = kops.linear(x, w)
    for N2, K2 in ((6144, 4096), (4096, 14336), (128, 64)):
        kops.linear(torch.randn(M, K2, device="cuda").bfloat16(), torch.randn(N2, K2, device="cuda").bfloat16())
    b = kops.linear(x, w)
    assert torch.equal(a, b)
    assert kops.check_status() == 0


@pytest.mark.parametrize("M,N,K", [(48, 4096, 4096), (5, 2048, 14336), (128, 1024, 2048)])
def test_gemm_scale_and_pre(kops, M, N, K):
    """The mixture epilogue: x . w^T * scale[m] + pre (+ residual), split and unsplit tiles."""
    g = torch.Generator(device="cuda").manual_seed(M + N)
    x = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    w = (torch.randn(N, K, device="cuda", generator=g) / math.sqrt(K)).bfloat16()
    scale = torch.rand(M, device="cuda", generator=g)
    pre = torch.randn(M, N, device="cuda", generator=g).bfloat16()
    r = torch.randn(M, N, device="cuda", generator=g).bfloat16()
    y = kops.linear(x, w, residual=r, scale=scale, pre=pre)
    close(y, ref.linear(x, w, None, r, scale, pre))
    y2 = kops.linear(x, w, scale=scale)
    close(y2, (x.float() @ w.float().t()) * scale[:, None])
    assert kops.check_status() == 0


@pytest.mark.parametrize("E,k,e0,el", [(8, 2, 0, 8), (8, 2, 4, 2), (64, 6, 8, 16), (4, 1, 1, 3)])
def test_moe_route(kops, E, k, e0, el):
    g = torch.Generator(device="cuda").manual_seed(E * 10 + k)
    logits = (torch.randn(37, E, device="cuda", generator=g) * 2).bfloat16()
    got = kops.moe_route(logits, k, e0, el)
    want = ref.moe_route(logits, k, e0, el)
    assert torch.equal(got > 0, want > 0)
    torch.testing.assert_close(got, want, rtol=1e-5, atol=1e-6)


def test_gemm_batch_invariant(kops):
    """A row's result does not depend on the other rows of the batch (exact replay needs this)."""
    g = torch.Generator(device="cuda").manual_seed(4)
    N, K = 4096, 4096
    w = (torch.randn(N, K, device="cuda", generator=g) / 64).bfloat16()
    x = torch.randn(64, K, device="cuda", generator=g).bfloat16()
    full = kops.linear(x, w)
    for m in (1, 3, 17, 40):
        part = kops.linear(x[:m].contiguous(), w)
        assert torch.equal(part, full[:m]), f"rows differ at M={m}"


@pytest.mark.parametrize("hq,hkv,d,bs", [(32, 8, 128, 16), (4, 1, 128, 16), (14, 2, 64, 16), (64, 8, 128, 32),
                                         (8, 8, 64, 32)])
def test_paged_decode(kops, decode_kernel, hq, hkv, d, bs):
    g = torch.Generator(device="cuda").manual_seed(5)
    lens = [1, 15, 16, 17, 64, 255, 256, 257, 700, 1029]
    B = len(lens)
    max_len = 1100
    mb = (max_len + bs - 1) // bs
    nb = B * mb + 3
    cache = torch.randn(nb, 2, hkv, bs, d, device="cuda", generator=g).bfloat16()
    perm = torch.randperm(nb, device="cuda", generator=g)[: B * mb].view(B, mb).int()
    ctx = torch.tensor(lens, device="cuda", dtype=torch.int32)
    q = torch.randn(B, hq, d, device="cuda", generator=g).bfloat16()
    scale = 1 / math.sqrt(d)
    out = kops.decode_attention(q, cache, perm, ctx, scale, max_len)
    seq = torch.arange(B, device="cuda")
    expect = ref.paged_attention(q.float(), cache.float(), perm, ctx, seq, ctx.long() - 1, scale)
    close(out, expect, rtol=2e-2, atol=2e-2)
    assert kops.check_status() == 0
    # batch invariance: one sequence alone gives the same bits
    one = kops.decode_attention(q[7:8].contiguous(), cache, perm[7:8].contiguous(), ctx[7:8].contiguous(), scale,
                                max_len)
    assert torch.equal(one, out[7:8])


@pytest.fixture(params=[0, 1], ids=["split", "persistent"])
def decode_kernel(request, kops):
    """Each decode-attention kernel in turn (the persistent one by its run-time switch)."""
    prev = kops.C.set_decode_persist(request.param)
    yield request.param
    kops.C.set_decode_persist(prev)


@pytest.mark.parametrize("hq,hkv,d,bs", [(32, 8, 128, 16), (64, 8, 64, 32), (8, 1, 128, 16)])
def test_paged_decode_ranges(kops, decode_kernel, hq, hkv, d, bs):
    """Many more (sequence, kv head, split) items than SMs, so the persistent kernel's ranges cut
    pairs (merged by the last range, one ticket per pair) as well as hold whole ones (merged in
    place): every output matches the fp32 oracle, sub-batches give the same bits, and a second call
    (tickets left at zero by the first) gives the same bits again. One history spans several
    ranges; empty histories give zero. The split kernel passes the same checks."""
    g = torch.Generator(device="cpu").manual_seed(11)
    B = 96
    lens = torch.randint(1, 3000, (B,), generator=g)
    lens[3] = 0
    lens[40] = 0
    lens[50] = 24000
    lens[51] = 1
    max_len = 24064
    mb = (max_len + bs - 1) // bs
    need = [int((n + bs - 1) // bs) for n in lens.tolist()]
    nb = sum(need) + 8
    cache = torch.randn(nb, 2, hkv, bs, d, generator=g).bfloat16().cuda()
    perm = torch.randperm(nb, generator=g)
    bt = torch.zeros(B, mb, dtype=torch.int32)
    used = 0
    for b, k in enumerate(need):
        bt[b, :k] = perm[used:used + k].int()
        used += k
    bt = bt.cuda()
    ctx = lens.int().cuda()
    q = torch.randn(B, hq, d, generator=g).bfloat16().cuda()
    scale = 1 / math.sqrt(d)
    out = kops.decode_attention(q, cache, bt, ctx, scale, max_len)
    assert kops.check_status() == 0
    live = [b for b in range(B) if lens[b] > 0]
    idx = torch.tensor(live, device="cuda")
    expect = ref.paged_attention(q[idx].float(), cache.float(), bt[idx], ctx[idx], torch.arange(len(live), device="cuda"),
                                 ctx[idx].long() - 1, scale)
    close(out[idx], expect, rtol=2e-2, atol=2e-2)
    assert torch.count_nonzero(out[3]) == 0 and torch.count_nonzero(out[40]) == 0
    again = kops.decode_attention(q, cache, bt, ctx, scale, max_len)
    assert torch.equal(again, out)
    for lo, hi in ((50, 51), (0, 7), (45, 60), (90, 96)):
        part = kops.decode_attention(q[lo:hi].contiguous(), cache, bt[lo:hi].contiguous(), ctx[lo:hi].contiguous(),
                                     scale, max_len)
        assert torch.equal(part, out[lo:hi]), f"rows {lo}:{hi} depend on the batch"
    assert kops.check_status() == 0


def test_kv_gather_scatter(kops):
    C = kops.C
    g = torch.Generator(device="cuda").manual_seed(6)
    L, nb, hkv, bs, d = 3, 10, 4, 16, 128
    caches = [torch.randn(nb, 2, hkv, bs, d, device="cuda", generator=g).bfloat16() for _ in range(L)]
    ptrs = torch.tensor([c.data_ptr() for c in caches], device="cuda", dtype=torch.int64)
    slots = torch.tensor([5, 17, -1, 100, 159], device="cuda")
    heads = torch.tensor([1, 3], device="cuda")
    cap = 8
    staging = torch.full((L, 2, cap, 2, d), 7.0, device="cuda").bfloat16()
    strides = [caches[0].stride(i) for i in (0, 3, 2, 1, 4)]
    C.kv_gather(ptrs, slots, heads, staging.data_ptr(), cap, d, bs, strides, 2)
    for l in range(L):
        for hi, h in enumerate([1, 3]):
            for t, s in enumerate(slots.tolist()):
                if s < 0:
                    assert torch.count_nonzero(staging[l, hi, t]) == 0
                    continue
                assert torch.equal(staging[l, hi, t, 0], caches[l][s // bs, 0, h, s % bs])
                assert torch.equal(staging[l, hi, t, 1], caches[l][s // bs, 1, h, s % bs])
    # scatter into zeroed caches restores exactly those rows
    fresh = [torch.zeros_like(c) for c in caches]
    ptrs2 = torch.tensor([c.data_ptr() for c in fresh], device="cuda", dtype=torch.int64)
    C.kv_scatter(ptrs2, slots, heads, staging.data_ptr(), cap, d, bs, strides, 2)
    for l in range(L):
        for h in (1, 3):
            for s in slots.tolist():
                if s >= 0:
                    assert torch.equal(fresh[l][s // bs, :, h, s % bs], caches[l][s // bs, :, h, s % bs])
        assert torch.count_nonzero(fresh[l][:, :, 0]) == 0


def test_kv_gather_to_mapped_host(kops):
    """The gather writes straight into pinned, device-mapped host memory (the store's rows)."""
    C = kops.C
    L, nb, hkv, bs, d, cap = 2, 4, 2, 16, 64, 4
    caches = [torch.randn(nb, 2, hkv, bs, d, device="cuda").bfloat16() for _ in range(L)]
    ptrs = torch.tensor([c.data_ptr() for c in caches], device="cuda", dtype=torch.int64)
    host = torch.zeros(L * hkv * cap * 2 * d, dtype=torch.bfloat16)
    dev_ptr = C.host_register_mapped(host.data_ptr(), host.numel() * 2)
    try:
        slots = torch.tensor([0, 33, 63], device="cuda")
        heads = torch.arange(hkv, device="cuda")
        C.kv_gather(ptrs, slots, heads, dev_ptr, cap, d, bs, [caches[0].stride(i) for i in (0, 3, 2, 1, 4)], 2)
        torch.cuda.synchronize()
        view = host.view(L, hkv, cap, 2, d)
        assert torch.equal(view[1, 1, 1, 0], caches[1][33 // bs, 0, 1, 33 % bs].cpu())
    finally:
        C.host_unregister(host.data_ptr())


@pytest.mark.parametrize("M,N,K", [(64, 28672, 4096), (5, 3584, 4096), (1, 256, 512), (33, 9728, 896), (200, 3584, 4096)])
def test_gemm_silu_fused(kops, M, N, K):
    """SiLU-mul in the GEMM epilogue (gate/up rows interleaved by 64) equals the GEMM followed by the
    SiLU-mul kernel bit for bit, and the fp32 oracle within bf16 tolerance."""
    from everserve_b200.ops import interleave_gate_up

    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    x = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    gu = (torch.randn(N, K, device="cuda", generator=g) / math.sqrt(K)).bfloat16()
    w = interleave_gate_up(gu).contiguous()
    fused = kops.linear_silu(x, w)
    unfused = kops.silu_mul(kops.linear(x, w), interleaved=True)
    assert torch.equal(fused, unfused)
    # (the plain layout puts a row in another tile, so its k-blocks split differently: close, not equal)
    close(unfused, kops.silu_mul(kops.linear(x, gu)))
    gate, up = (x.float() @ gu.float().t()).chunk(2, dim=1)
    close(fused, torch.nn.functional.silu(gate) * up)
    assert kops.check_status() == 0


def test_gemm_stream_k_repeats_and_tail(kops):
    """Stream-K: runs that end inside a tile park partials for the CTA that finishes the tile; the
    result does not change over repeated launches (epoch flags) or with the token count."""
    g = torch.Generator(device="cuda").manual_seed(9)
    for N, K in ((128256 // 8, 4096), (4096, 14336), (1000, 1792), (128, 64), (6144, 4096)):
        w = (torch.randn(N, K, device="cuda", generator=g) / math.sqrt(K)).bfloat16()
        x = torch.randn(64, K, device="cuda", generator=g).bfloat16()
        first = kops.linear(x, w)
        for _ in range(3):
            assert torch.equal(kops.linear(x, w), first)
        assert torch.equal(kops.linear(x[:7].contiguous(), w), first[:7])
        close(first, x.float() @ w.float().t())
    assert kops.check_status() == 0


@pytest.mark.parametrize("M,N,K", [(64, 28672, 4096), (64, 4096, 14336), (7, 1000, 1792), (200, 3584, 4096),
                                   (64, 128, 64)])
def test_gemm_packed_weights(kops, M, N, K):
    """A weight kept as its packed stage blocks (one bulk copy per stage) gives the tiled weight's
    result bit for bit: the same tiles, k-blocks and order, only the loads differ. The packed
    blocks round-trip to the weight; the fused SiLU-mul and residual epilogues take them too."""
    from everserve_b200.ops import PackedWeight, interleave_gate_up

    g = torch.Generator(device="cuda").manual_seed(M * 7 + N + K)
    x = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    w = (torch.randn(N, K, device="cuda", generator=g) / math.sqrt(K)).bfloat16()
    pw = PackedWeight(w)
    assert torch.equal(pw.unpack(), w)
    assert torch.equal(kops.linear(x, pw), kops.linear(x, w))
    r = torch.randn(M, N, device="cuda", generator=g).bfloat16()
    assert torch.equal(kops.linear(x, pw, residual=r), kops.linear(x, w, residual=r))
    close(kops.linear(x, pw), x.float() @ w.float().t())
    if N % 128 == 0 and M <= 64:
        wi = interleave_gate_up(w).contiguous()
        assert torch.equal(kops.linear_silu(x, PackedWeight(wi)), kops.linear_silu(x, wi))
    assert kops.check_status() == 0


@pytest.mark.parametrize("T,hq,hkv,packed", [(64, 32, 8, False), (7, 8, 2, True), (130, 16, 4, False)])
def test_gemm_rope_kv_epilogue(kops, T, hq, hkv, packed):
    """The qkv GEMM with RoPE and the paged-KV write in its epilogue gives q and the cache rows of
    the separate GEMM + rope_kv_write kernels (the same bf16-rounded product, rotated by the same
    table) to within one bf16 rounding, and leaves every other cache row untouched."""
    from everserve_b200.ops import PackedWeight, ref

    g = torch.Generator(device="cuda").manual_seed(T + hq)
    d, bs, K = 128, 16, 1024
    x = torch.randn(T, K, device="cuda", generator=g).bfloat16()
    w = (torch.randn((hq + 2 * hkv) * d, K, device="cuda", generator=g) / math.sqrt(K)).bfloat16()
    pos = torch.randint(0, 4000, (T,), device="cuda", generator=g)
    cs = ref.cos_sin_table(d, 4096, 5e5).cuda()
    nb = T // bs + 8
    slots = torch.randperm(nb * bs, device="cuda", generator=g)[:T]
    slots[0] = -1  # a padding row: q only
    c_fused = torch.randn(nb, 2, hkv, bs, d, device="cuda", generator=g).bfloat16()
    c_plain = c_fused.clone()
    q_fused = kops.linear_rope_kv(x, PackedWeight(w) if packed else w, pos, cs, slots, c_fused, hq, hkv, bs)
    q_plain = kops.rope_kv_write(kops.linear(x, w), None, pos, cs, slots, c_plain, hq, hkv, bs)
    torch.cuda.synchronize()
    assert kops.check_status() == 0

    def ulps(a, b):  # distance in bf16 steps
        ia = a.contiguous().view(torch.int16).int()
        ib = b.contiguous().view(torch.int16).int()
        return (ia - ib).abs().max().item()

    assert ulps(q_fused, q_plain) <= 1
    assert ulps(c_fused, c_plain) <= 1
    # untouched rows are bit-identical (the padding row's slot included)
    written = torch.zeros(nb * bs, dtype=torch.bool, device="cuda")
    written[slots[slots >= 0]] = True
    keep = ~written.view(nb, bs)
    assert torch.equal(c_fused.permute(0, 3, 1, 2, 4)[keep], c_plain.permute(0, 3, 1, 2, 4)[keep])
