"""Hugging Face checkpoints round-trip into model shards (TP1 and TP2, dense and MoE)."""

import torch
from safetensors.torch import save_file

from everserve_b200.models.config import get_config
from everserve_b200.models.llama import DecoderLM, TPGroup
from everserve_b200.models.weights import load_hf_checkpoint, to_hf_state_dict


def _roundtrip(name, tmp_path):
    cfg = get_config(name)
    full = DecoderLM(cfg, "cpu", torch.float32, seed=5)
    save_file(to_hf_state_dict(full), str(tmp_path / "model.safetensors"))
    same = DecoderLM(cfg, "cpu", torch.float32, seed=99, init="none")
    load_hf_checkpoint(same, str(tmp_path))
    assert set(same.weights) == set(full.weights)
    for k in full.weights:
        assert torch.equal(same.weights[k], full.weights[k]), k
    # a tensor-parallel shard of the checkpoint is the random-init shard of the same seed
    for r in range(2):
        shard = DecoderLM(cfg, "cpu", torch.float32, seed=99, tp=TPGroup(r, 2), init="none")
        load_hf_checkpoint(shard, str(tmp_path))
        ref = DecoderLM(cfg, "cpu", torch.float32, seed=5, tp=TPGroup(r, 2))
        for k in ref.weights:
            assert torch.equal(shard.weights[k], ref.weights[k]), (r, k)


def test_llama_checkpoint_roundtrip(tmp_path):
    _roundtrip("tiny-llama", tmp_path)


def test_qwen_checkpoint_roundtrip(tmp_path):
    _roundtrip("tiny-qwen", tmp_path)


def test_mixtral_checkpoint_roundtrip(tmp_path):
    _roundtrip("tiny-mixtral", tmp_path)


def test_engine_serves_a_checkpoint(tmp_path):
    """An engine started from a checkpoint generates what the model it was exported from does."""
    from everserve_b200.engine.config import EngineConfig
    from everserve_b200.engine.engine import Engine

    cfg = get_config("tiny-qwen")
    save_file(to_hf_state_dict(DecoderLM(cfg, "cpu", torch.float32, seed=7)), str(tmp_path / "model.safetensors"))
    prompts = [[1, 2, 3, 4], [9, 8, 7]]
    a = Engine(EngineConfig("tiny-qwen", device="cpu", dtype=torch.float32, seed=7, num_blocks=32, max_batch=4,
                            max_model_len=64)).generate(prompts, max_tokens=6)
    b = Engine(EngineConfig("tiny-qwen", device="cpu", dtype=torch.float32, seed=123, num_blocks=32, max_batch=4,
                            max_model_len=64, checkpoint=str(tmp_path))).generate(prompts, max_tokens=6)
    assert a == b
