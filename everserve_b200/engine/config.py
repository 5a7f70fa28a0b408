"""Engine configuration."""

from __future__ import annotations

import os
from dataclasses import dataclass, field

import torch

from ..models.config import ModelConfig, get_config


@dataclass
class EngineConfig:
    model: ModelConfig | str
    device: str = "cuda"
    dtype: torch.dtype = torch.bfloat16
    seed: int = 0
    block_size: int = 16
    num_blocks: int | None = None  # None: fill `kv_memory_fraction` of the free device memory
    kv_memory_fraction: float = 0.85
    max_batch: int = 64
    max_model_len: int = 4096
    max_prefill_tokens: int = 8192
    tensor_parallel: int = 1
    pipeline_parallel: int = 1
    use_cuda_graphs: bool = True
    checkpoint: str | None = None  # a Hugging Face safetensors directory; None: random-init from `seed`
    # "fp8": the dense projections' weights in e4m3 with one scale per 128 x 128 block, activations
    # quantized per token and 128-wide block (the block-scaled fp8 GEMM); None: bf16
    quant: str | None = None
    # tensor-parallel ranks keep the residual stream of their token slice (norms on the slice,
    # reduce-scatter GEMMs for o/down, all-gather GEMMs for qkv/gate_up/vocabulary); ES_SP=1 sets it
    sequence_parallel: bool = field(default_factory=lambda: os.environ.get("ES_SP", "0") == "1")
    # mixture models on the GPU kernels: prefill-size steps route tokens to their experts (within
    # the GPU, or to the experts' owners over a peer-memory TP group) instead of running every
    # local expert on every token; ES_MOE_ROUTED=0 turns it off
    moe_routed: bool = field(default_factory=lambda: os.environ.get("ES_MOE_ROUTED", "1") != "0")
    # Engine.step keeps one decode step in flight: step N+1 is enqueued (its token fed from step N's
    # sampled id on the device) before step N's ids are read back, so the host's bookkeeping overlaps
    # the device; ES_ASYNC_DECODE=0 turns it off
    async_decode: bool = field(default_factory=lambda: os.environ.get("ES_ASYNC_DECODE", "1") != "0")
    extra: dict = field(default_factory=dict)

    def __post_init__(self):
        if isinstance(self.model, str):
            self.model = get_config(self.model)
        if self.block_size not in (16, 32):
            raise ValueError("block_size must be 16 or 32")
        if self.quant not in (None, "fp8"):
            raise ValueError(f"unknown quantization {self.quant!r}")

    @property
    def world_size(self) -> int:
        return self.tensor_parallel * self.pipeline_parallel
