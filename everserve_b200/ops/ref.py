"""PyTorch reference implementations of every decoder op.

These are the arithmetic of the CPU engine (fp32 on CPU, the reference tier and the
CPU/gloo configuration) and the numerical oracle of the sm_100a kernels: each kernel's test
compares against the function here evaluated in fp32.

Conventions shared with the kernels:
  * RMSNorm: ``y = x * rsqrt(mean(x^2) + eps) * w`` in fp32, one rounding to the output dtype;
    with a residual, ``r = round(x + r)`` is stored first and then normalised.
  * RoPE: rotate-half pairs (i, i + d/2), angles from a precomputed fp32 ``cos_sin`` table
    ``[max_pos, d]`` holding cos in the first half and sin in the second.
  * KV cache of one layer: ``[num_blocks, 2, kv_heads, block_size, head_dim]``; slot = block *
    block_size + offset; a negative slot is a padding token and is not written.

Reference parity: HF-convention rms_norm / rope / llama3 inverse frequencies of
core/everserve/reference/arith/ops.py:17-73.
"""

from __future__ import annotations

import math

import torch


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, residual: torch.Tensor | None = None) -> torch.Tensor:
    if residual is not None:
        s = (x.float() + residual.float()).to(residual.dtype)
        residual.copy_(s)
        x = s
    xf = x.float()
    inv = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (xf * inv * w.float()).to(x.dtype)


def inverse_frequencies(head_dim: int, theta: float, scaling: dict | None = None) -> torch.Tensor:
    """Rotary inverse frequencies, with the llama3 long-context scaling when ``scaling`` asks."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))
    if scaling and scaling.get("rope_type", scaling.get("type")) == "llama3":
        factor = scaling["factor"]
        lo, hi = scaling.get("low_freq_factor", 1.0), scaling.get("high_freq_factor", 4.0)
        old_ctx = scaling.get("original_max_position_embeddings", 8192)
        lo_wl, hi_wl = old_ctx / lo, old_ctx / hi
        wl = 2 * math.pi / inv
        smooth = (old_ctx / wl - lo) / (hi - lo)
        scaled = torch.where(wl > lo_wl, inv / factor, inv)
        mid = (wl <= lo_wl) & (wl >= hi_wl)
        scaled = torch.where(mid, (1 - smooth) * inv / factor + smooth * inv, scaled)
        inv = scaled
    return inv.float()


def cos_sin_table(head_dim: int, max_pos: int, theta: float, scaling: dict | None = None) -> torch.Tensor:
    inv = inverse_frequencies(head_dim, theta, scaling).double()
    ang = torch.arange(max_pos, dtype=torch.float64)[:, None] * inv[None, :]
    return torch.cat([torch.cos(ang), torch.sin(ang)], dim=-1).float()


def rope(x: torch.Tensor, cs: torch.Tensor) -> torch.Tensor:
    """x: [T, H, d] (fp32), cs: [T, d] cos|sin rows for each token."""
    half = x.shape[-1] // 2
    c, s = cs[:, None, :half], cs[:, None, half:]
    a, b = x[..., :half], x[..., half:]
    return torch.cat([a * c - b * s, b * c + a * s], dim=-1)


def rope_kv_write(qkv, bias, positions, cos_sin, slots, cache, hq: int, hkv: int, block_size: int) -> torch.Tensor:
    """Rotate q and k, write k and v into the paged cache; return q as [T, hq, d]."""
    T = qkv.shape[0]
    d = cos_sin.shape[1]
    x = qkv.float()
    if bias is not None:
        x = x + bias.float()
    x = x.view(T, hq + 2 * hkv, d)
    cs = cos_sin[positions]
    q = rope(x[:, :hq], cs)
    k = rope(x[:, hq : hq + hkv], cs)
    v = x[:, hq + hkv :]
    valid = slots >= 0
    if bool(valid.any()):
        sl = slots[valid]
        blk, off = sl // block_size, sl % block_size
        cache[blk, 0, :, off] = k[valid].to(cache.dtype)
        cache[blk, 1, :, off] = v[valid].to(cache.dtype)
    return q.to(qkv.dtype)


def gather_kv(cache: torch.Tensor, block_table: torch.Tensor, n: int) -> tuple[torch.Tensor, torch.Tensor]:
    """The first n positions of one sequence: k, v as [n, kv_heads, d]."""
    bs = cache.shape[3]
    nb = (n + bs - 1) // bs
    blocks = cache[block_table[:nb].long()]  # [nb, 2, Hkv, bs, d]
    k = blocks[:, 0].permute(0, 2, 1, 3).reshape(nb * bs, cache.shape[2], cache.shape[4])[:n]
    v = blocks[:, 1].permute(0, 2, 1, 3).reshape(nb * bs, cache.shape[2], cache.shape[4])[:n]
    return k, v


def paged_attention(q, cache, block_tables, ctx_lens, q_seq, q_pos, scale: float) -> torch.Tensor:
    """Causal attention of query rows against their sequence's paged history.

    q: [T, hq, d]; q_seq[t] is the row's sequence index into block_tables/ctx_lens, q_pos[t] its
    position (it sees positions 0..q_pos[t]). Returns [T, hq, d] in q's dtype (fp32 inside).
    """
    T, hq, d = q.shape
    hkv = cache.shape[2]
    g = hq // hkv
    out = torch.empty_like(q)
    seqs = q_seq.tolist()
    pos = q_pos.tolist()
    start = 0
    while start < T:
        s = seqs[start]
        end = start
        while end < T and seqs[end] == s:
            end += 1
        n = int(ctx_lens[s])
        k, v = gather_kv(cache, block_tables[s], n)
        kf = k.float().repeat_interleave(g, dim=1)  # [n, hq, d]
        vf = v.float().repeat_interleave(g, dim=1)
        qf = q[start:end].float()
        scores = torch.einsum("thd,nhd->htn", qf, kf) * scale
        p_idx = torch.tensor(pos[start:end], device=q.device)
        mask = torch.arange(n, device=q.device)[None, :] > p_idx[:, None]
        scores = scores.masked_fill(mask[None], float("-inf"))
        prob = torch.softmax(scores, dim=-1)
        out[start:end] = torch.einsum("htn,nhd->thd", prob, vf).to(q.dtype)
        start = end
    return out


def silu_mul(gu: torch.Tensor) -> torch.Tensor:
    inter = gu.shape[-1] // 2
    g, u = gu[..., :inter].float(), gu[..., inter:].float()
    return (g * torch.sigmoid(g) * u).to(gu.dtype)


def linear(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None,
           residual: torch.Tensor | None = None, scale: torch.Tensor | None = None,
           pre: torch.Tensor | None = None) -> torch.Tensor:
    """x . w^T * scale[m] + pre + bias + residual (fp32, one rounding): the GEMM epilogue's order."""
    y = x.float() @ w.float().t()
    if scale is not None:
        y = y * scale.float()[:, None]
    if pre is not None:
        y = y + pre.float()
    if bias is not None:
        y = y + bias.float()
    if residual is not None:
        y = y + residual.float()
    return y.to(x.dtype)


def moe_route(logits: torch.Tensor, k: int, e0: int, el: int) -> torch.Tensor:
    """Per-token weights of experts e0 .. e0 + el - 1: softmax, top k with ties to the lowest index,
    renormalised over the k; 0 for an expert not chosen. Returns fp32 [el, T]."""
    p = torch.softmax(logits.float(), dim=-1)
    order = torch.argsort(-p, dim=-1, stable=True)[:, :k]
    chosen = torch.zeros_like(p).scatter_(1, order, 1.0)
    w = p * chosen / (p * chosen).sum(-1, keepdim=True)
    return w[:, e0 : e0 + el].t().contiguous()


def moe_topk(logits: torch.Tensor, k: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Each token's top k experts by softmax probability (ties to the lowest index), in rank
    order, and their probabilities renormalised over the k: (int32 [T, k], fp32 [T, k])."""
    p = torch.softmax(logits.float(), dim=-1)
    ids = torch.argsort(-p, dim=-1, stable=True)[:, :k]
    w = p.gather(1, ids)
    return ids.to(torch.int32), w / w.sum(-1, keepdim=True)


def expert_places(ids: torch.Tensor, num_experts: int) -> torch.Tensor:
    """Where each (token, slot) row goes in its expert's segment from this sender: its rank among
    the sender's rows for the same expert in (token, slot) order. int32 like `ids`."""
    flat = ids.reshape(-1).long()
    onehot = torch.nn.functional.one_hot(flat, num_experts)
    before = onehot.cumsum(0) - onehot  # rows of each expert strictly before this one
    return before.gather(1, flat[:, None]).reshape(ids.shape).to(torch.int32)


def moe_a2a(xs: list[torch.Tensor], ids: list[torch.Tensor], weights: list[torch.Tensor], expert) -> list[torch.Tensor]:
    """Oracle of the expert-parallel all-to-all: for each member's tokens x [T, H], the sum over
    slots (in order, fp32) of weight * expert(e, x[t]); `expert(e, rows)` gives fp32 outputs."""
    outs = []
    for x, i, w in zip(xs, ids, weights):
        acc = torch.zeros(x.shape, dtype=torch.float32, device=x.device)
        for j in range(i.shape[1]):
            for e in i[:, j].unique().tolist():
                rows = (i[:, j] == e).nonzero().flatten()
                acc[rows] += w[rows, j, None].float() * expert(int(e), x[rows]).float()
        outs.append(acc.to(x.dtype))
    return outs


def argmax(logits: torch.Tensor) -> torch.Tensor:
    return torch.argmax(logits.float(), dim=-1)


def member_sum(parts: list[torch.Tensor]) -> torch.Tensor:
    """Sum of the members' tensors in member order, fp32 accumulate, one rounding.

    The oracle of the failure-detecting all-reduce: the same order after a membership change
    gives the same bits (core/everserve/reference/arith/ops.py:63).
    """
    acc = torch.zeros_like(parts[0], dtype=torch.float32)
    for p in parts:
        acc = acc + p.float()
    return acc.to(parts[0].dtype)
