"""Placement-independent decoder arithmetic: outputs bit-identical whichever rank owns which unit.

A rank owns units of two kinds: attention units (one KV head with the query heads that share it)
and MLP units (fixed-width slices of the intermediate dimension, or chunks of experts for a
mixture). Each layer, every owned unit writes its partial output (its heads' slice of o_proj, its
slice of down_proj) into its own slot of a ``[units, tokens, hidden]`` fp32 buffer that is zero
elsewhere; the buffer is summed over the ranks (a sum of one non-zero and zeros is exact), and
every rank then adds the slots in unit order. The shapes a unit computes with never depend on the
placement, so the result is the same before and after a loss: when a rank dies, the survivors
``absorb`` its units (load their weights, restore their heads' KV from the committed store) and
continue with identical outputs. This is the SHRINK outcome.

KV caches here are contiguous per (layer, attention unit, sequence): the tier is a specification,
not a paged engine.

Reference parity: the placement-independent cores of core/everserve/reference/arith/cores.py:46-443
(ReferenceCore, LlamaCore with fixed-width MLP slices, the MoE core with fixed expert chunks,
absorb); the arithmetic here is this framework's.
"""

from __future__ import annotations

from typing import Callable, Sequence

import torch

from ..models.config import ModelConfig
from .arith import DeterministicSource, cos_sin_table, rmsnorm, rope


class LlamaCore:
    """A dense (or top-k mixture) decoder whose work is split into movable units."""

    def __init__(self, cfg: ModelConfig, rank: int, attn_units: Sequence[int], mlp_units: Sequence[int],
                 n_mlp_units: int, source=None, reduce: Callable[[torch.Tensor], torch.Tensor] | None = None,
                 max_pos: int = 4096):
        self.cfg, self.rank = cfg, rank
        self.src = source or DeterministicSource(0)
        self.reduce = reduce or (lambda t: t)
        self.hq, self.hkv, self.d, self.H = cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.hidden
        self.G = self.hq // self.hkv
        self.n_mlp = n_mlp_units
        if cfg.num_experts:
            if cfg.num_experts % n_mlp_units:
                raise ValueError("experts must split into equal chunks")
        elif cfg.intermediate % n_mlp_units:
            raise ValueError("the intermediate dimension must split into equal slices")
        self.cs = cos_sin_table(self.d, max_pos, cfg.rope_theta, cfg.rope_scaling)
        self.scale = self.d ** -0.5
        L, H, V = cfg.layers, self.H, cfg.vocab
        self.embed = self.src.get("embed", (V, H))
        self.lm_head = self.embed if cfg.tie_embeddings else self.src.get("lm_head", (V, H))
        self.final_norm = 1.0 + self.src.get("final_norm", (H,))
        self.in_norm = [1.0 + self.src.get(f"l{l}.in_norm", (H,)) for l in range(L)]
        self.post_norm = [1.0 + self.src.get(f"l{l}.post_norm", (H,)) for l in range(L)]
        if cfg.num_experts:
            self.router = [self.src.get(f"l{l}.router", (cfg.num_experts, H)) for l in range(L)]
        self.attn: dict[int, dict] = {}
        self.mlp: dict[int, dict] = {}
        self.kv: dict[tuple[int, int, int], torch.Tensor] = {}  # (layer, kv head, seq) -> [n, 2, d]
        self.load_units(attn_units, mlp_units)

    # ---- units -----------------------------------------------------------------------------------
    def _attn_weights(self, u: int) -> dict:
        d, G, H = self.d, self.G, self.H
        w = {}
        for l in range(self.cfg.layers):
            w[(l, "q")] = torch.cat([self.src.get(f"l{l}.q.h{u * G + g}", (d, H)) for g in range(G)])
            w[(l, "k")] = self.src.get(f"l{l}.k.h{u}", (d, H))
            w[(l, "v")] = self.src.get(f"l{l}.v.h{u}", (d, H))
            w[(l, "o")] = torch.cat([self.src.get(f"l{l}.o.h{u * G + g}", (H, d)) for g in range(G)], dim=1)
        return w

    def _mlp_weights(self, m: int) -> dict:
        c, H = self.cfg, self.H
        w = {}
        if c.num_experts:
            per = c.num_experts // self.n_mlp
            for l in range(c.layers):
                for e in range(m * per, (m + 1) * per):
                    w[(l, e, "g")] = self.src.get(f"l{l}.e{e}.g", (c.intermediate, H))
                    w[(l, e, "u")] = self.src.get(f"l{l}.e{e}.u", (c.intermediate, H))
                    w[(l, e, "d")] = self.src.get(f"l{l}.e{e}.d", (H, c.intermediate))
            return w
        width = c.intermediate // self.n_mlp
        for l in range(c.layers):
            w[(l, "g")] = self.src.get(f"l{l}.g.s{m}", (width, H))
            w[(l, "u")] = self.src.get(f"l{l}.u.s{m}", (width, H))
            w[(l, "d")] = self.src.get(f"l{l}.d.s{m}", (H, width))
        return w

    def load_units(self, attn_units: Sequence[int], mlp_units: Sequence[int]) -> None:
        for u in attn_units:
            if u not in self.attn:
                self.attn[u] = self._attn_weights(u)
        for m in mlp_units:
            if m not in self.mlp:
                self.mlp[m] = self._mlp_weights(m)

    def absorb(self, attn_units: Sequence[int], mlp_units: Sequence[int], kv_rows: dict) -> None:
        """Take over units of a lost rank: their weights, and their heads' committed KV rows
        (`kv_rows`: (layer, kv head, seq) -> [n, 2, d])."""
        self.load_units(attn_units, mlp_units)
        for key, rows in kv_rows.items():
            if key[1] in set(attn_units):
                self.kv[key] = rows.clone()

    def mark(self) -> dict:
        """The KV lengths now (rolled back to by ``rollback`` when an attempt is abandoned)."""
        return {k: v.shape[0] for k, v in self.kv.items()}

    def rollback(self, mark: dict) -> None:
        for k in list(self.kv):
            n = mark.get(k)
            if n is None:
                del self.kv[k]
            elif self.kv[k].shape[0] != n:
                self.kv[k] = self.kv[k][:n].clone()

    # ---- the forward ---------------------------------------------------------------------------
    def _slots_sum(self, parts: dict[int, torch.Tensor], n_units: int, T: int) -> torch.Tensor:
        buf = torch.zeros(n_units, T, self.H)
        for u, p in parts.items():
            buf[u] = p
        buf = self.reduce(buf)
        out = buf[0].clone()
        for u in range(1, n_units):
            out = out + buf[u]
        return out

    def forward(self, ids: torch.Tensor, positions: torch.Tensor, seqs: torch.Tensor) -> tuple[torch.Tensor, dict]:
        """One step for tokens `ids` at `positions` of sequences `seqs` (each sequence's tokens in
        position order). Returns the logits of every token and the KV rows this rank wrote
        ((layer, kv head, seq) -> [n, 2, d]) for the committed store."""
        c, T = self.cfg, ids.shape[0]
        h = self.embed[ids].clone()
        cs = self.cs[positions]
        written: dict[tuple[int, int, int], list] = {}
        for l in range(c.layers):
            x = rmsnorm(h, self.in_norm[l], c.rms_eps)
            parts = {}
            for u, w in self.attn.items():
                q = rope((x @ w[(l, "q")].t()).view(T, self.G, self.d), cs)
                k = rope((x @ w[(l, "k")].t()).view(T, 1, self.d), cs)[:, 0]
                v = x @ w[(l, "v")].t()
                o = torch.empty(T, self.G, self.d)
                for sq in seqs.unique(sorted=True).tolist():
                    idx = (seqs == sq).nonzero()[:, 0]
                    new = torch.stack([k[idx], v[idx]], dim=1)  # [n, 2, d]
                    key = (l, u, sq)
                    past = self.kv.get(key)
                    cache = new if past is None else torch.cat([past, new])
                    self.kv[key] = cache
                    written.setdefault(key, []).append(new)
                    n_new, n_all = idx.numel(), cache.shape[0]
                    s = torch.einsum("tgd,nd->tgn", q[idx], cache[:, 0]) * self.scale
                    causal = torch.arange(n_all)[None, :] <= (n_all - n_new + torch.arange(n_new))[:, None]
                    s = s.masked_fill(~causal[:, None, :], float("-inf"))
                    o[idx] = torch.einsum("tgn,nd->tgd", torch.softmax(s, dim=-1), cache[:, 1])
                parts[u] = o.reshape(T, self.G * self.d) @ w[(l, "o")].t()
            h = h + self._slots_sum(parts, self.hkv, T)
            x = rmsnorm(h, self.post_norm[l], c.rms_eps)
            parts = {}
            if c.num_experts:
                probs = torch.softmax(x @ self.router[l].t(), dim=-1)
                topv, topi = torch.topk(probs, c.top_k, dim=-1)
                topv = topv / topv.sum(-1, keepdim=True)
                per = c.num_experts // self.n_mlp
                for m, w in self.mlp.items():
                    acc = torch.zeros(T, self.H)
                    for e in range(m * per, (m + 1) * per):
                        gate = (topv * (topi == e)).sum(-1)  # [T]
                        y = torch.nn.functional.silu(x @ w[(l, e, "g")].t()) * (x @ w[(l, e, "u")].t())
                        acc = acc + gate[:, None] * (y @ w[(l, e, "d")].t())
                    parts[m] = acc
            else:
                for m, w in self.mlp.items():
                    a = torch.nn.functional.silu(x @ w[(l, "g")].t()) * (x @ w[(l, "u")].t())
                    parts[m] = a @ w[(l, "d")].t()
            h = h + self._slots_sum(parts, self.n_mlp, T)
        logits = rmsnorm(h, self.final_norm, c.rms_eps) @ self.lm_head.t()
        return logits, {k: torch.cat(v) for k, v in written.items()}
