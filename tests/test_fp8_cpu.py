"""The fp8 configuration on the CPU engine: the dense projections' weights are block-scaled e4m3
(128 x 128 blocks), the activations quantized per token and block, and a generation runs through
the same engine with logits close to the bf16 model's."""

import torch

from everserve_b200.engine import Engine, EngineConfig
from everserve_b200.models.config import TINY_LLAMA
from everserve_b200.models.llama import DecoderLM, StepInput
from everserve_b200.ops import dequantize_fp8


def _logits(model, prompt):
    T = len(prompt)
    bs = 16
    cache = [torch.zeros(model.kv_cache_shape(8, bs), dtype=model.dtype) for _ in range(model.cfg.layers)]
    inp = StepInput(ids=torch.tensor(prompt), positions=torch.arange(T), slots=torch.arange(T),
                    block_tables=torch.arange(8, dtype=torch.int32)[None], ctx_lens=torch.tensor([T], dtype=torch.int32),
                    q_seq=torch.zeros(T, dtype=torch.int64), logits_idx=torch.tensor([T - 1]), is_decode=False)
    return model.logits(inp, cache)


def test_fp8_weights_are_block_quantized_and_close():
    bf = DecoderLM(TINY_LLAMA, "cpu", torch.float32, seed=3)
    f8 = DecoderLM(TINY_LLAMA, "cpu", torch.float32, seed=3, quant="fp8")
    q, s = f8.weights["l0.qkv.q8"], f8.weights["l0.qkv.s8"]
    assert q.dtype == torch.float8_e4m3fn and s.shape == ((q.shape[0] + 127) // 128, q.shape[1] // 128)
    assert "l0.qkv" not in f8.weights and "l0.in_norm" in f8.weights
    w = bf.weights["l0.qkv"]
    assert (dequantize_fp8(q, s, 128) - w).abs().max() <= w.abs().max() / 16
    prompt = [5, 17, 99, 3, 250, 7]
    a, b = _logits(bf, prompt), _logits(f8, prompt)
    assert ((a - b).norm() / a.norm()) < 0.1


def test_fp8_engine_generates():
    eng = Engine(EngineConfig(TINY_LLAMA, device="cpu", dtype=torch.float32, max_batch=4, max_model_len=128,
                              num_blocks=32, quant="fp8"))
    out = eng.generate([[1, 2, 3, 4], [9, 8, 7]], max_tokens=5)
    assert [len(o) for o in out] == [5, 5]
