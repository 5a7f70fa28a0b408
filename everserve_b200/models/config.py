"""Model architectures the engine serves, with the shapes of the benchmark configurations.

Every model is a pre-norm decoder (RMSNorm, RoPE, GQA attention, SwiGLU MLP or a top-k softmax
mixture of SwiGLU experts). Weights are random-initialised from a seed (no checkpoints are
available offline); ``load_hf_checkpoint`` in :mod:`everserve_b200.models.weights` reads real ones.
"""

from __future__ import annotations

from dataclasses import asdict, dataclass, field


@dataclass(frozen=True)
class ModelConfig:
    name: str
    vocab: int
    hidden: int
    layers: int
    heads: int
    kv_heads: int
    head_dim: int
    intermediate: int
    rope_theta: float = 10000.0
    rms_eps: float = 1e-6
    tie_embeddings: bool = False
    qkv_bias: bool = False
    num_experts: int = 0  # 0: dense MLP
    top_k: int = 2
    max_position: int = 8192
    rope_scaling: dict | None = field(default=None, hash=False, compare=False)

    @property
    def is_moe(self) -> bool:
        return self.num_experts > 0

    def params(self) -> int:
        attn = self.hidden * (self.heads + 2 * self.kv_heads) * self.head_dim + self.heads * self.head_dim * self.hidden
        mlp = 3 * self.hidden * self.intermediate * max(1, self.num_experts)
        router = self.hidden * self.num_experts
        emb = self.vocab * self.hidden * (1 if self.tie_embeddings else 2)
        return self.layers * (attn + mlp + router + 2 * self.hidden) + emb + self.hidden

    def to_dict(self) -> dict:
        return asdict(self)


QWEN2_5_0_5B = ModelConfig(
    name="qwen2.5-0.5b", vocab=151936, hidden=896, layers=24, heads=14, kv_heads=2, head_dim=64,
    intermediate=4864, rope_theta=1e6, rms_eps=1e-6, tie_embeddings=True, qkv_bias=True, max_position=32768,
)

LLAMA3_8B = ModelConfig(
    name="llama-3-8b", vocab=128256, hidden=4096, layers=32, heads=32, kv_heads=8, head_dim=128,
    intermediate=14336, rope_theta=5e5, rms_eps=1e-5, max_position=8192,
)

LLAMA3_70B = ModelConfig(
    name="llama-3-70b", vocab=128256, hidden=8192, layers=80, heads=64, kv_heads=8, head_dim=128,
    intermediate=28672, rope_theta=5e5, rms_eps=1e-5, max_position=8192,
)

MIXTRAL_8X7B = ModelConfig(
    name="mixtral-8x7b", vocab=32000, hidden=4096, layers=32, heads=32, kv_heads=8, head_dim=128,
    intermediate=14336, rope_theta=1e6, rms_eps=1e-5, num_experts=8, top_k=2, max_position=32768,
)

# small shapes for tests (same structure, fewer and narrower layers)
TINY_LLAMA = ModelConfig(
    name="tiny-llama", vocab=512, hidden=256, layers=2, heads=4, kv_heads=2, head_dim=64,
    intermediate=512, rope_theta=1e4, rms_eps=1e-5, max_position=2048,
)
TINY_QWEN = ModelConfig(
    name="tiny-qwen", vocab=512, hidden=256, layers=4, heads=4, kv_heads=2, head_dim=64,
    intermediate=256, rope_theta=1e6, rms_eps=1e-6, tie_embeddings=True, qkv_bias=True, max_position=2048,
)
TINY_MIXTRAL = ModelConfig(
    name="tiny-mixtral", vocab=512, hidden=256, layers=2, heads=4, kv_heads=2, head_dim=64,
    intermediate=256, rope_theta=1e6, rms_eps=1e-5, num_experts=4, top_k=2, max_position=2048,
)

# a small model whose tensor-parallel shards still meet the GPU kernels' tile sizes (TP <= 4)
SMALL_LLAMA = ModelConfig(
    name="small-llama", vocab=4096, hidden=1024, layers=4, heads=16, kv_heads=8, head_dim=64,
    intermediate=2048, rope_theta=5e5, rms_eps=1e-5, max_position=4096,
)

REGISTRY = {c.name: c for c in (QWEN2_5_0_5B, LLAMA3_8B, LLAMA3_70B, MIXTRAL_8X7B, TINY_LLAMA, TINY_QWEN, TINY_MIXTRAL,
                                SMALL_LLAMA)}


def get_config(name: str) -> ModelConfig:
    try:
        return REGISTRY[name]
    except KeyError:
        raise KeyError(f"unknown model {name!r}; known: {sorted(REGISTRY)}") from None
