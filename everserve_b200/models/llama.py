"""The pre-norm decoder (Llama 3, Qwen2, Mixtral) with tensor- and pipeline-parallel sharding.

One instance holds one rank's shard: the layers of its pipeline stage, and within each layer its
tensor-parallel slice (column-parallel qkv/gate_up, row-parallel o/down whose partial outputs the
collective sums, vocab-parallel embedding/lm_head). MoE layers shard their experts across the
tensor-parallel group (expert parallelism over the same ranks).

Weights are random-initialised: each full parameter is drawn from a generator seeded by (seed,
layer, name) and then sliced, so a rank's shard is the same tensor whoever builds it. A spare that
takes rank r builds exactly rank r's weights.

Arithmetic goes through an op set (``everserve_b200.ops``): the sm_100a kernels on CUDA, the
PyTorch reference on CPU. The row-parallel linears call ``linear_allreduce`` of the tensor-parallel
group, which is the fused GEMM + all-reduce when the group has one.
"""

from __future__ import annotations

import hashlib
import os
from dataclasses import dataclass

import torch

from ..ops import PackedWeight, interleave_gate_up, ops_for, quantize_weight_fp8, ref, softmax_scale
from .config import ModelConfig


@dataclass
class StepInput:
    """One forward's inputs (all on the model's device)."""

    ids: torch.Tensor  # [T] int64 token ids (stage 0)
    positions: torch.Tensor  # [T] int64
    slots: torch.Tensor  # [T] int64 cache slots (-1 = padding)
    block_tables: torch.Tensor  # [B, max_blocks] int32
    ctx_lens: torch.Tensor  # [B] int32: context length after this step's tokens
    q_seq: torch.Tensor  # [T] int64: sequence index of each row
    logits_idx: torch.Tensor  # [B] int64: each sequence's last row
    is_decode: bool
    max_model_len: int = 0
    sampling: object | None = None  # engine.sampling.SamplingBatch of the rows; None: greedy
    logprobs_k: int | None = None  # the step also reports log-probabilities (k alternatives)
    prefill_tiles: torch.Tensor | None = None  # prefill kernel work list (ops.prefill_tiles), device


def _seed_of(seed: int, *parts) -> int:
    h = hashlib.sha256(repr((seed,) + parts).encode()).digest()
    return int.from_bytes(h[:8], "little") & ((1 << 63) - 1)


class TPGroup:
    """Tensor-parallel context of one rank. Size 1 needs no collective."""

    def __init__(self, rank: int = 0, size: int = 1, collective=None):
        self.rank, self.size, self.collective = rank, size, collective

    def all_reduce(self, t: torch.Tensor) -> torch.Tensor:
        if self.size == 1:
            return t
        return self.collective.all_reduce(t)

    def linear_allreduce(self, ops, x, w, residual=None, scale=None, pre=None, prefetch=None):
        """Row-parallel linear (x . w^T * scale + pre) followed by the sum over ranks, then the
        residual; one fused kernel when the collective has it. `prefetch`: what the next kernel
        reads, fetched into L2 meanwhile (kernels only)."""
        if self.size == 1:
            return ops.linear(x, w, residual=residual, scale=scale, pre=pre, prefetch=prefetch)
        fused = getattr(self.collective, "linear_allreduce", None)
        if fused is not None and ops.kind == "kernel":
            if getattr(self.collective, "region", None) is not None:  # the peer-memory collective
                return fused(ops, x, w, residual, scale=scale, pre=pre, prefetch=prefetch)
            return fused(ops, x, w, residual, scale=scale, pre=pre)
        y = self.collective.all_reduce(ops.linear(x, w, scale=scale, pre=pre))
        if residual is not None:
            y = (y.float() + residual.float()).to(y.dtype)
        return y

    def all_gather_rows(self, t: torch.Tensor) -> torch.Tensor:
        """Concatenate each rank's [*, n] tensor along the last dim (rank order)."""
        if self.size == 1:
            return t
        return self.collective.all_gather(t)

    # ---- the sequence-parallel pair: token slices between the projections ----------------------
    def token_slice(self, M: int) -> tuple[int, int, int]:
        """(per, first, last): this rank keeps tokens [first, last) of M, per = ceil(M / size)."""
        per = -(-M // self.size)
        return per, min(M, self.rank * per), min(M, (self.rank + 1) * per)

    def gather_rows(self, t: torch.Tensor) -> torch.Tensor:
        """Every rank's [per, K] rows, in rank order: [per * size, K]."""
        if self.size == 1:
            return t
        flat = self.collective.all_gather(t.reshape(1, -1).contiguous())
        return flat.reshape(self.size * t.shape[0], t.shape[1])

    def gather_linear(self, ops, x_local, w):
        """Column-parallel linear over every rank's token rows (rank order): [per * size, N]; the
        all-gather fused into the GEMM when the collective has it."""
        if self.size == 1:
            return ops.linear(x_local, w)
        fused = getattr(self.collective, "gather_linear", None)
        if fused is not None and ops.kind == "kernel":
            return fused(ops, x_local, w)
        return ops.linear(self.gather_rows(x_local), w)

    def reduce_scatter_linear(self, ops, x, w):
        """Row-parallel linear whose sum over the ranks this rank keeps for its token slice only:
        [per, N] (rows past the tokens are padding); fused into the GEMM when the collective has it."""
        if self.size == 1:
            return ops.linear(x, w)
        fused = getattr(self.collective, "linear_reduce_scatter", None)
        if fused is not None and ops.kind == "kernel":
            return fused(ops, x, w)
        y = self.collective.all_reduce(ops.linear(x, w))
        per, lo, hi = self.token_slice(x.shape[0])
        out = torch.zeros(per, y.shape[1], dtype=y.dtype, device=y.device)
        out[: hi - lo] = y[lo:hi]
        return out


class DecoderLM:
    # the dense projections that take block-scaled fp8 weights in the fp8 configuration
    FP8_LINEARS = ("qkv", "o", "gate_up", "down")
    # the dense projections whose weights the kernels keep packed in stage blocks (one bulk copy per
    # stage streams them front to back; measured faster for the large MLP matrices at decode)
    PACKED_LINEARS = ("gate_up", "down")

    def __init__(self, cfg: ModelConfig, device="cpu", dtype=torch.bfloat16, seed: int = 0,
                 tp: TPGroup | None = None, layer_range: tuple[int, int] | None = None,
                 init: str = "random", quant: str | None = None, sequence_parallel: bool = False):
        self.cfg = cfg
        # fp8: those weights stored as e4m3 with 128 x 128 block scales (key.q8, key.s8)
        self.fp8 = quant == "fp8"
        if self.fp8 and cfg.is_moe:
            raise ValueError("the fp8 configuration covers dense models")
        self.device = torch.device(device)
        self.dtype = dtype
        self.seed = seed
        self.step_logprobs = None  # the last forward's log-probabilities, when it was asked for them
        self.a2a = None  # routed experts (parallel.moe_a2a), when enabled
        self.tp = tp or TPGroup()
        self.ops = ops_for(self.device)
        self.l0, self.l1 = layer_range or (0, cfg.layers)
        self.first = self.l0 == 0
        self.last = self.l1 == cfg.layers
        # token-sliced residual stream between the projections (one stage, dense, bf16 weights)
        self.sequence_parallel = bool(sequence_parallel) and self.tp.size > 1
        if self.sequence_parallel and (cfg.is_moe or quant or not (self.first and self.last)):
            raise ValueError("sequence parallelism covers single-stage dense bf16 models")
        T, r = self.tp.size, self.tp.rank
        assert cfg.heads % T == 0, "query heads must divide by the tensor-parallel size"
        self.hq = cfg.heads // T
        if cfg.kv_heads >= T:
            assert cfg.kv_heads % T == 0
            self.hkv = cfg.kv_heads // T
            self.kv_head0 = r * self.hkv
        else:  # fewer kv heads than ranks: replicate
            assert T % cfg.kv_heads == 0
            self.hkv = 1
            self.kv_head0 = r * cfg.kv_heads // T
        self.d = cfg.head_dim
        self.scale = softmax_scale(cfg.head_dim)
        if cfg.is_moe:
            assert cfg.num_experts % T == 0, "experts must divide by the expert-parallel size"
            self.experts_local = cfg.num_experts // T
            self.expert0 = r * self.experts_local
            self.inter = cfg.intermediate
        else:
            assert cfg.intermediate % T == 0
            self.inter = cfg.intermediate // T
        self.vocab_local = (cfg.vocab + T - 1) // T
        self.vocab0 = r * self.vocab_local
        # dense gate_up weights on the kernels are stored interleaved by 64 rows, so the decode GEMM
        # computes SiLU-mul in its epilogue (ops.linear_silu); the reference ops keep gate then up
        self.fused_silu = (not cfg.is_moe and self.ops.kind == "kernel" and self.inter % 64 == 0
                           and os.environ.get("ES_FUSED_SILU", "1") != "0")
        # the qkv GEMM's RoPE + KV-write epilogue (kernels, bf16, head dim 128, no qkv bias)
        self.fused_rope = (self.ops.kind == "kernel" and not self.fp8 and cfg.head_dim == 128
                           and not cfg.qkv_bias and os.environ.get("ES_FUSED_ROPE", "1") != "0")
        self.packed_weights = (self.ops.kind == "kernel" and not cfg.is_moe
                               and os.environ.get("ES_PACK_WEIGHTS", "1") != "0")
        self.cos_sin = ref.cos_sin_table(cfg.head_dim, cfg.max_position, cfg.rope_theta, cfg.rope_scaling).to(self.device)
        self.weights: dict[str, torch.Tensor] = {}
        if init == "random":
            self._init_random()

    # ---- weights -----------------------------------------------------------------------------
    def _rand(self, name: str, layer: int, shape, std: float = 0.02) -> torch.Tensor:
        gen_dev = self.device if self.device.type == "cuda" else torch.device("cpu")
        g = torch.Generator(device=gen_dev)
        g.manual_seed(_seed_of(self.seed, layer, name))
        t = torch.randn(*shape, generator=g, device=gen_dev, dtype=torch.float32) * std
        return t

    def _put(self, key: str, t: torch.Tensor):
        if self.fused_silu and key.endswith(".gate_up") and ".e" not in key:
            t = interleave_gate_up(t)
        if self.fp8 and key.rsplit(".", 1)[-1] in self.FP8_LINEARS:
            q, s = quantize_weight_fp8(t.to(device=self.device, dtype=torch.float32))
            self.weights[key + ".q8"], self.weights[key + ".s8"] = q.contiguous(), s.contiguous()
            return
        t = t.to(device=self.device, dtype=self.dtype).contiguous()
        if self.packed_weights and key.rsplit(".", 1)[-1] in self.PACKED_LINEARS and ".e" not in key:
            self.weights[key] = PackedWeight(t)  # the packed blocks only; ops.dense(w) unpacks
            return
        self.weights[key] = t

    def _linear(self, ops, x, key: str, residual=None):
        """x . W[key]^T (+ residual) for a bf16 or a block-scaled fp8 weight."""
        if self.fp8:
            return ops.linear_fp8(x, self.weights[key + ".q8"], self.weights[key + ".s8"], residual)
        return ops.linear(x, self.weights[key], residual=residual)

    def _row_parallel(self, ops, x, key: str, residual=None, prefetch=None):
        """A row-parallel projection summed over the tensor-parallel ranks, then the residual."""
        if not self.fp8:
            return self.tp.linear_allreduce(ops, x, self.weights[key], residual, prefetch=prefetch)
        if self.tp.size == 1:
            return self._linear(ops, x, key, residual)
        y = self.tp.all_reduce(self._linear(ops, x, key))
        return y if residual is None else (y.float() + residual.float()).to(y.dtype)

    def _init_random(self):
        c, d = self.cfg, self.cfg.head_dim
        H = c.hidden
        qs = slice(self.tp.rank * self.hq * d, (self.tp.rank + 1) * self.hq * d)
        ks = slice(self.kv_head0 * d, (self.kv_head0 + self.hkv) * d)
        ones = torch.ones(H)
        if self.first or (self.last and c.tie_embeddings):
            emb = self._rand("embed", -1, (c.vocab, H))
            self._put("embed", self._vocab_slice(emb))
        for l in range(self.l0, self.l1):
            p = f"l{l}."
            q = self._rand("q", l, (c.heads * d, H))[qs]
            k = self._rand("k", l, (c.kv_heads * d, H))[ks]
            v = self._rand("v", l, (c.kv_heads * d, H))[ks]
            self._put(p + "qkv", torch.cat([q, k, v], 0))
            if c.qkv_bias:
                bq = self._rand("bq", l, (c.heads * d,), 0.1)[qs]
                bk = self._rand("bk", l, (c.kv_heads * d,), 0.1)[ks]
                bv = self._rand("bv", l, (c.kv_heads * d,), 0.1)[ks]
                self._put(p + "qkv_bias", torch.cat([bq, bk, bv]))
            self._put(p + "o", self._rand("o", l, (H, c.heads * d))[:, qs])
            self._put(p + "in_norm", ones)
            self._put(p + "post_norm", ones)
            if c.is_moe:
                self._put(p + "router", self._rand("router", l, (c.num_experts, H)))
                for e in range(self.expert0, self.expert0 + self.experts_local):
                    g_ = self._rand(f"gate{e}", l, (c.intermediate, H))
                    u_ = self._rand(f"up{e}", l, (c.intermediate, H))
                    self._put(p + f"e{e}.gate_up", torch.cat([g_, u_], 0))
                    self._put(p + f"e{e}.down", self._rand(f"down{e}", l, (H, c.intermediate)))
            else:
                ms = slice(self.tp.rank * self.inter, (self.tp.rank + 1) * self.inter)
                g_ = self._rand("gate", l, (c.intermediate, H))[ms]
                u_ = self._rand("up", l, (c.intermediate, H))[ms]
                self._put(p + "gate_up", torch.cat([g_, u_], 0))
                self._put(p + "down", self._rand("down", l, (H, c.intermediate))[:, ms])
        if self.last:
            self._put("final_norm", ones)
            if not c.tie_embeddings:
                self._put("lm_head", self._vocab_slice(self._rand("lm_head", -1, (c.vocab, H))))

    def _vocab_slice(self, t: torch.Tensor) -> torch.Tensor:
        s = t[self.vocab0 : self.vocab0 + self.vocab_local]
        if s.shape[0] < self.vocab_local:  # pad the last shard
            s = torch.cat([s, torch.zeros(self.vocab_local - s.shape[0], t.shape[1], device=t.device, dtype=t.dtype)])
        return s

    def linear_shapes(self) -> list[tuple[int, int]]:
        """(N, K) of every weight the forward multiplies by, for scratch sizing."""
        out = set()
        for k, w in self.weights.items():
            if w.dim() == 2 and k not in ("embed",):
                out.add((w.shape[0], w.shape[1]))
        if "embed" in self.weights and self.last and self.cfg.tie_embeddings:
            out.add(tuple(self.weights["embed"].shape))
        return sorted(out)

    # ---- KV cache ------------------------------------------------------------------------------
    def kv_cache_shape(self, num_blocks: int, block_size: int) -> tuple[int, ...]:
        return (num_blocks, 2, self.hkv, block_size, self.d)

    def bytes_per_block(self, block_size: int) -> int:
        return 2 * self.hkv * block_size * self.d * torch.tensor([], dtype=self.dtype).element_size() * (self.l1 - self.l0)

    # ---- forward -------------------------------------------------------------------------------
    def embed(self, ids: torch.Tensor) -> torch.Tensor:
        ops = self.ops
        if self.tp.size == 1:
            return ops.embed(ids, self.weights["embed"])
        # vocab-parallel: each rank looks up the ids in its slice, the sum over ranks fills the rest
        local = ids - self.vocab0
        mine = (local >= 0) & (local < self.vocab_local)
        x = ops.embed(torch.where(mine, local, torch.zeros_like(local)), self.weights["embed"])
        x = x * mine[:, None].to(x.dtype)
        return self.tp.all_reduce(x)

    def forward(self, inp: StepInput, caches: list[torch.Tensor], hidden: torch.Tensor | None = None,
                residual: torch.Tensor | None = None):
        """Run this stage. Returns (hidden, residual) for a middle stage, next-token ids for the last."""
        if self.sequence_parallel:
            return self._forward_sp(inp, caches)
        ops, c, W = self.ops, self.cfg, self.weights
        if self.first:
            x = self.embed(inp.ids)
            residual = x
            h = ops.rmsnorm(x, W[f"l{self.l0}.in_norm"], c.rms_eps)
        else:
            h = ops.rmsnorm(hidden, W[f"l{self.l0}.in_norm"], c.rms_eps, residual)
        bs = caches[0].shape[3] if caches else 16
        for i, l in enumerate(range(self.l0, self.l1)):
            p = f"l{l}."
            cache = caches[i]
            if self.fused_rope:
                # one kernel: the qkv GEMM rotates q and k and writes k and v to the cache
                q = ops.linear_rope_kv(h, W[p + "qkv"], inp.positions, self.cos_sin, inp.slots, cache,
                                       self.hq, self.hkv, bs)
            else:
                qkv = self._linear(ops, h, p + "qkv")
                q = ops.rope_kv_write(qkv, W.get(p + "qkv_bias"), inp.positions, self.cos_sin, inp.slots, cache,
                                      self.hq, self.hkv, bs)
            if inp.is_decode:
                if ops.kind == "kernel":
                    # the attention streams the history; meanwhile it brings o_proj's weights into L2
                    a = ops.decode_attention(q, cache, inp.block_tables, inp.ctx_lens, self.scale,
                                             inp.max_model_len or None, prefetch=W.get(p + "o"))
                else:
                    a = ops.decode_attention(q, cache, inp.block_tables, inp.ctx_lens, self.scale)
            else:
                a = ops.prefill_attention(q, cache, inp.block_tables, inp.ctx_lens, inp.q_seq, inp.positions,
                                          self.scale, inp.prefill_tiles)
            a = a.reshape(a.shape[0], self.hq * self.d)
            o = self._row_parallel(ops, a, p + "o")
            h = ops.rmsnorm(o, W[p + "post_norm"], c.rms_eps, residual)
            if c.is_moe:
                m = self._moe(h, p)
            else:
                if self.fp8:
                    act = ops.linear_fp8(h, W[p + "gate_up.q8"], W[p + "gate_up.s8"], silu=self.fused_silu)
                    if not self.fused_silu:
                        act = ops.silu_mul(act)
                elif self.fused_silu:
                    act = ops.linear_silu(h, W[p + "gate_up"])
                else:
                    act = ops.silu_mul(ops.linear(h, W[p + "gate_up"]))
                # decode: the down projection brings the next layer's qkv weights into L2
                pf = W.get(f"l{l + 1}.qkv") if inp.is_decode and l + 1 < self.l1 else None
                m = self._row_parallel(ops, act, p + "down", prefetch=pf)
            nxt = f"l{l + 1}.in_norm" if l + 1 < self.l1 else None
            if nxt is not None:
                h = ops.rmsnorm(m, W[nxt], c.rms_eps, residual)
            else:
                hidden = m
        if not self.last:
            return hidden, residual
        h = ops.rmsnorm(hidden, W["final_norm"], c.rms_eps, residual)
        h_last = h.index_select(0, inp.logits_idx) if h.shape[0] != inp.logits_idx.shape[0] else h
        head = W["embed"] if c.tie_embeddings else W["lm_head"]
        logits = ops.linear(h_last, head)
        ids = self._sample(logits, inp) if inp.sampling is not None else self._greedy(logits)
        if inp.logprobs_k is not None:
            self.step_logprobs = self._logprobs(logits, ids, inp.logprobs_k)
        return ids

    def _forward_sp(self, inp: StepInput, caches: list[torch.Tensor]):
        """The sequence-parallel forward: each rank keeps the residual stream of its slice of the
        step's tokens and runs the norms there; the column-parallel projections (qkv, gate_up, the
        vocabulary) take every rank's normalised rows through the all-gather fused into their GEMM,
        the row-parallel ones (o, down) reduce-scatter their sums by tokens in their GEMM's epilogue.
        Attention still sees every token of the rank's heads. The bytes on the links equal the
        all-reduce forward's; the norms and residual adds run on a 1/size slice, and each collective
        overlaps its own GEMM's weight streaming."""
        ops, c, W = self.ops, self.cfg, self.weights
        M = inp.ids.shape[0]
        per, lo, hi = self.tp.token_slice(M)
        x = self.embed(inp.ids)
        residual = torch.zeros(per, c.hidden, dtype=x.dtype, device=x.device)
        residual[: hi - lo] = x[lo:hi]
        h = ops.rmsnorm(residual, W[f"l{self.l0}.in_norm"], c.rms_eps)
        bs = caches[0].shape[3] if caches else 16
        hidden = None
        for i, l in enumerate(range(self.l0, self.l1)):
            p = f"l{l}."
            cache = caches[i]
            qkv = self.tp.gather_linear(ops, h, W[p + "qkv"])[:M]  # the first M rows: contiguous
            q = ops.rope_kv_write(qkv, W.get(p + "qkv_bias"), inp.positions, self.cos_sin, inp.slots, cache,
                                  self.hq, self.hkv, bs)
            if inp.is_decode:
                if ops.kind == "kernel":
                    # the attention streams the history; meanwhile it brings o_proj's weights into L2
                    a = ops.decode_attention(q, cache, inp.block_tables, inp.ctx_lens, self.scale,
                                             inp.max_model_len or None, prefetch=W.get(p + "o"))
                else:
                    a = ops.decode_attention(q, cache, inp.block_tables, inp.ctx_lens, self.scale)
            else:
                a = ops.prefill_attention(q, cache, inp.block_tables, inp.ctx_lens, inp.q_seq, inp.positions,
                                          self.scale, inp.prefill_tiles)
            a = a.reshape(M, self.hq * self.d)
            o = self.tp.reduce_scatter_linear(ops, a, W[p + "o"])
            h = ops.rmsnorm(o, W[p + "post_norm"], c.rms_eps, residual)
            gu = self.tp.gather_linear(ops, h, W[p + "gate_up"])[:M].contiguous()
            act = ops.silu_mul(gu, interleaved=self.fused_silu)
            m = self.tp.reduce_scatter_linear(ops, act, W[p + "down"])
            if l + 1 < self.l1:
                h = ops.rmsnorm(m, W[f"l{l + 1}.in_norm"], c.rms_eps, residual)
            else:
                hidden = m
        h = ops.rmsnorm(hidden, W["final_norm"], c.rms_eps, residual)
        head = W["embed"] if c.tie_embeddings else W["lm_head"]
        if inp.is_decode and M <= 64 and inp.logits_idx.shape[0] == M:
            logits = self.tp.gather_linear(ops, h, head)[:M]
        else:
            rows = self.tp.gather_rows(h)[:M]
            logits = ops.linear(rows.index_select(0, inp.logits_idx), head)
        ids = self._sample(logits, inp) if inp.sampling is not None else self._greedy(logits)
        if inp.logprobs_k is not None:
            self.step_logprobs = self._logprobs(logits, ids, inp.logprobs_k)
        return ids

    def _logprobs(self, logits: torch.Tensor, ids: torch.Tensor, k: int):
        """Each row's chosen token's log-probability and its k most likely tokens with theirs
        (the model's distribution, before temperature and filters): ([B], [B, k], [B, k])."""
        full = logits if self.tp.size == 1 else self.tp.all_gather_rows(logits.contiguous())
        lsm = torch.log_softmax(full[:, : self.cfg.vocab].float(), dim=-1)
        chosen = lsm.gather(1, ids.view(-1, 1).long())[:, 0]
        top = torch.topk(lsm, max(0, min(k, lsm.shape[1])), dim=-1)
        return chosen, top.indices, top.values

    def _sample(self, logits: torch.Tensor, inp: StepInput) -> torch.Tensor:
        """Seeded sampling of every row (engine.sampling); each tensor-parallel rank gathers the
        full vocabulary and draws the same tokens."""
        full = logits if self.tp.size == 1 else self.tp.all_gather_rows(logits.contiguous())
        full = full[:, : self.cfg.vocab]
        pos = inp.positions if inp.positions.shape[0] == full.shape[0] else inp.positions.index_select(0, inp.logits_idx)
        return self.ops.sample(full, pos, inp.sampling)

    def logits(self, inp: StepInput, caches, hidden=None, residual=None):
        """Full-vocab logits of each sequence's last row (tests and the CPU oracle)."""
        saved = self._greedy
        out = {}

        def grab(lg):
            out["l"] = lg
            return saved(lg)

        self._greedy = grab
        try:
            self.forward(inp, caches, hidden, residual)
        finally:
            self._greedy = saved
        lg = out["l"]
        if self.tp.size > 1:
            lg = self.tp.all_gather_rows(lg.contiguous())
        return lg[:, : self.cfg.vocab]

    def _greedy(self, logits: torch.Tensor) -> torch.Tensor:
        ops = self.ops
        if self.tp.size == 1:
            return ops.argmax(logits[:, : self.cfg.vocab] if logits.shape[1] != self.cfg.vocab else logits)
        # vocab-parallel greedy: local (value, index) pairs, gathered, best value then lowest index
        idx = ops.argmax(logits)
        val = logits.gather(1, idx[:, None]).float()
        valid_n = min(self.vocab_local, self.cfg.vocab - self.vocab0)
        val = torch.where(idx[:, None] < valid_n, val, torch.full_like(val, float("-inf")))
        pair = torch.cat([val, (idx + self.vocab0).float()[:, None]], dim=1)  # [B, 2]
        allp = self.tp.all_gather_rows(pair.contiguous()).view(pair.shape[0], self.tp.size, 2)
        best = allp[:, :, 0].argmax(dim=1)  # first rank holding the max value = lowest index
        return allp[torch.arange(pair.shape[0], device=pair.device), best, 1].long()

    # ---- MoE -----------------------------------------------------------------------------------
    def enable_routed_experts(self, max_tokens: int) -> bool:
        """Route each token to its experts' owners instead of running every local expert on every
        token (``parallel.moe_a2a``): rank r takes the r-th slice of the step's (replicated) tokens,
        the all-to-all carries each row to the ranks owning its top k experts, the experts run
        grouped GEMMs over what they received (tiles no token reached are skipped: unchosen experts
        read no weights, and prefill does the routed FLOPs instead of E/k times them), the combine
        brings the weighted outputs back, and an all-gather of the slices replicates the result.
        On one GPU the same kernels route within the GPU (a group of one, buffers in its own
        memory). Needs the GPU kernels and, across GPUs, a peer-memory collective; False (nothing
        changes) otherwise. Steps of at least ROUTED_MIN_TOKENS tokens (prefill) take the routed
        path; smaller ones (decode) keep running every local expert, which reads the same weight
        bytes and has no dispatch or combine."""
        if not self.cfg.is_moe or self.ops.kind != "kernel":
            return False
        from ..parallel.moe_a2a import ExpertAllToAll, default_cap

        if self.tp.size == 1:
            self.a2a = ExpertAllToAll.emulated(self.device, 1, experts=self.cfg.num_experts, top_k=self.cfg.top_k,
                                               hidden=self.cfg.hidden, cap=default_cap(max_tokens))
            return True
        coll = self.tp.collective
        if coll is None or not hasattr(coll, "region") or getattr(coll, "nvls", False):
            return False
        per = -(-max_tokens // self.tp.size)
        self.a2a = ExpertAllToAll.over(coll, experts=self.cfg.num_experts, top_k=self.cfg.top_k,
                                       hidden=self.cfg.hidden, cap=default_cap(per))
        return True

    # tokens from which a step routes them to their experts (prefill); ES_MOE_ROUTED_MIN overrides
    ROUTED_MIN_TOKENS = int(os.environ.get("ES_MOE_ROUTED_MIN", "512"))

    def _moe_routed(self, h: torch.Tensor, p: str) -> torch.Tensor:
        ops, c, W = self.ops, self.cfg, self.weights
        T, R = h.shape[0], self.tp.size
        if R == 1:
            logits = (h.float() @ W[p + "router"].float().t()).to(h.dtype)
            ids, weights = ops.moe_topk(logits, c.top_k)
            return self.a2a(ops, h.contiguous()[None], ids[None], weights[None], lambda e: W[p + f"e{e}.gate_up"],
                            lambda e: W[p + f"e{e}.down"])[0]
        per = -(-T // R)
        lo = min(T, self.tp.rank * per)
        hi = min(T, lo + per)
        mine = h[lo:hi].contiguous()
        logits = (mine.float() @ W[p + "router"].float().t()).to(h.dtype)
        ids, weights = ops.moe_topk(logits, c.top_k)
        out = self.a2a(ops, mine[None], ids[None], weights[None], lambda e: W[p + f"e{e}.gate_up"],
                       lambda e: W[p + f"e{e}.down"])[0]
        full = torch.zeros(R * per, h.shape[1], dtype=h.dtype, device=h.device)
        full[lo:hi] = out
        return self.tp.all_reduce(full)[:T]  # disjoint slices: the sum is the gather, exactly

    def _moe(self, h: torch.Tensor, p: str) -> torch.Tensor:
        """Top-k softmax mixture over this rank's experts, combined over the ranks.

        Tokens are replicated over the expert-parallel group (its attention is tensor-parallel), so
        dispatch is local: a routing kernel turns the router logits into each local expert's weight
        per token (0 for tokens not routed to it). Each expert runs on every token (a decode step
        reads each expert's weights once whatever the token count, so the extra rows cost no
        bandwidth) with its routing weight applied in the down projection's epilogue, and the
        experts of a rank accumulate in expert order through the epilogue's `pre` input. The last
        expert's down projection carries the combine over the ranks (the fused all-reduce). No host
        synchronisation, so the layer is captured in CUDA graphs; fixed orders, so results are
        deterministic.
        """
        if self.a2a is not None and h.shape[0] >= self.ROUTED_MIN_TOKENS:
            return self._moe_routed(h, p)
        ops, c, W = self.ops, self.cfg, self.weights
        # the router's product is a few experts wide: a plain matmul, not a weight-streaming GEMM
        logits = (h.float() @ W[p + "router"].float().t()).to(h.dtype)
        scales = ops.moe_route(logits, c.top_k, self.expert0, self.experts_local)
        acc = None
        for i, e in enumerate(range(self.expert0, self.expert0 + self.experts_local)):
            act = ops.silu_mul(ops.linear(h, W[p + f"e{e}.gate_up"]))
            if i == self.experts_local - 1:
                return self.tp.linear_allreduce(ops, act, W[p + f"e{e}.down"], scale=scales[i], pre=acc)
            acc = ops.linear(act, W[p + f"e{e}.down"], scale=scales[i], pre=acc)
        return acc
