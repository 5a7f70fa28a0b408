"""Real checkpoints: Hugging Face Llama / Qwen2 / Mixtral safetensors into a DecoderLM shard.

``load_hf_checkpoint(model, directory)`` reads the checkpoint's ``*.safetensors`` files and fills
the model's weights for its own shard (its layer range, its tensor-parallel slice of heads, MLP
columns, experts and vocabulary), in the model's fused layout: ``qkv`` (q, k, v rows stacked),
``gate_up`` (gate rows, then up rows), ``o`` / ``down`` column slices, ``e<i>.gate_up`` and
``e<i>.down`` per local expert, vocabulary-sliced ``embed`` / ``lm_head``. Rotary weights need no
permutation: the kernels use the rotate-half pairing of the Hugging Face format.

``to_hf_state_dict(model)`` is the inverse for a full (TP1, all layers) model: it writes the
model's weights under the Hugging Face names (used by tests, and to export random-init models).
"""

from __future__ import annotations

import glob
import os

import torch

from ..ops import deinterleave_gate_up, dense
from .llama import DecoderLM


def _names(directory: str) -> dict[str, str]:
    from safetensors import safe_open

    names = {}
    files = sorted(glob.glob(os.path.join(directory, "*.safetensors")))
    if not files:
        raise FileNotFoundError(f"no .safetensors files in {directory}")
    for path in files:
        with safe_open(path, framework="pt") as f:
            for k in f.keys():
                names[k] = path
    return names


class _Reader:
    def __init__(self, directory: str):
        from safetensors import safe_open

        self._names = _names(directory)
        self._open = safe_open
        self._handles = {}

    def has(self, name: str) -> bool:
        return name in self._names

    def get(self, name: str) -> torch.Tensor:
        path = self._names[name]
        if path not in self._handles:
            self._handles[path] = self._open(path, framework="pt")
        return self._handles[path].get_tensor(name)


def load_hf_checkpoint(model: DecoderLM, directory: str) -> None:
    c, d = model.cfg, model.cfg.head_dim
    rd = _Reader(directory)
    qs = slice(model.tp.rank * model.hq * d, (model.tp.rank + 1) * model.hq * d)
    ks = slice(model.kv_head0 * d, (model.kv_head0 + model.hkv) * d)
    if model.first or (model.last and c.tie_embeddings):
        model._put("embed", model._vocab_slice(rd.get("model.embed_tokens.weight").float()))
    for l in range(model.l0, model.l1):
        hf, p = f"model.layers.{l}.", f"l{l}."
        a = hf + "self_attn."
        q = rd.get(a + "q_proj.weight")[qs]
        k = rd.get(a + "k_proj.weight")[ks]
        v = rd.get(a + "v_proj.weight")[ks]
        model._put(p + "qkv", torch.cat([q, k, v], 0).float())
        if c.qkv_bias:
            b = [rd.get(a + f"{n}_proj.bias") for n in ("q", "k", "v")]
            model._put(p + "qkv_bias", torch.cat([b[0][qs], b[1][ks], b[2][ks]]).float())
        model._put(p + "o", rd.get(a + "o_proj.weight")[:, qs].float())
        model._put(p + "in_norm", rd.get(hf + "input_layernorm.weight").float())
        model._put(p + "post_norm", rd.get(hf + "post_attention_layernorm.weight").float())
        if c.is_moe:
            m = hf + "block_sparse_moe."
            model._put(p + "router", rd.get(m + "gate.weight").float())
            for e in range(model.expert0, model.expert0 + model.experts_local):
                ex = m + f"experts.{e}."
                model._put(p + f"e{e}.gate_up",
                           torch.cat([rd.get(ex + "w1.weight"), rd.get(ex + "w3.weight")], 0).float())
                model._put(p + f"e{e}.down", rd.get(ex + "w2.weight").float())
        else:
            ms = slice(model.tp.rank * model.inter, (model.tp.rank + 1) * model.inter)
            mlp = hf + "mlp."
            model._put(p + "gate_up", torch.cat([rd.get(mlp + "gate_proj.weight")[ms],
                                                 rd.get(mlp + "up_proj.weight")[ms]], 0).float())
            model._put(p + "down", rd.get(mlp + "down_proj.weight")[:, ms].float())
    if model.last:
        model._put("final_norm", rd.get("model.norm.weight").float())
        if not c.tie_embeddings:
            name = "lm_head.weight" if rd.has("lm_head.weight") else "model.embed_tokens.weight"
            model._put("lm_head", model._vocab_slice(rd.get(name).float()))


def to_hf_state_dict(model: DecoderLM) -> dict[str, torch.Tensor]:
    """The Hugging Face names of a full model's weights (TP1, every layer)."""
    if model.tp.size != 1 or not (model.first and model.last):
        raise ValueError("export needs the whole model in one shard")
    c, d = model.cfg, model.cfg.head_dim
    W = {k: dense(v).detach().float().cpu() for k, v in model.weights.items()}
    out = {"model.embed_tokens.weight": W["embed"][: c.vocab], "model.norm.weight": W["final_norm"]}
    if not c.tie_embeddings:
        out["lm_head.weight"] = W["lm_head"][: c.vocab]
    nq, nk = c.heads * d, c.kv_heads * d
    for l in range(c.layers):
        hf, p = f"model.layers.{l}.", f"l{l}."
        qkv = W[p + "qkv"]
        out[hf + "self_attn.q_proj.weight"] = qkv[:nq]
        out[hf + "self_attn.k_proj.weight"] = qkv[nq : nq + nk]
        out[hf + "self_attn.v_proj.weight"] = qkv[nq + nk :]
        if c.qkv_bias:
            b = W[p + "qkv_bias"]
            out[hf + "self_attn.q_proj.bias"], out[hf + "self_attn.k_proj.bias"] = b[:nq], b[nq : nq + nk]
            out[hf + "self_attn.v_proj.bias"] = b[nq + nk :]
        out[hf + "self_attn.o_proj.weight"] = W[p + "o"]
        out[hf + "input_layernorm.weight"] = W[p + "in_norm"]
        out[hf + "post_attention_layernorm.weight"] = W[p + "post_norm"]
        if c.is_moe:
            m = hf + "block_sparse_moe."
            out[m + "gate.weight"] = W[p + "router"]
            for e in range(c.num_experts):
                gu = W[p + f"e{e}.gate_up"]
                out[m + f"experts.{e}.w1.weight"], out[m + f"experts.{e}.w3.weight"] = gu[: c.intermediate], gu[c.intermediate :]
                out[m + f"experts.{e}.w2.weight"] = W[p + f"e{e}.down"]
        else:
            gu = W[p + "gate_up"]
            if getattr(model, "fused_silu", False):
                gu = deinterleave_gate_up(gu)
            out[hf + "mlp.gate_proj.weight"], out[hf + "mlp.up_proj.weight"] = gu[: c.intermediate], gu[c.intermediate :]
            out[hf + "mlp.down_proj.weight"] = W[p + "down"]
    return {k: v.clone().contiguous() for k, v in out.items()}
