"""Model definitions (pre-norm decoders: Llama 3, Qwen2, Mixtral)."""

from .config import LLAMA3_8B, LLAMA3_70B, MIXTRAL_8X7B, QWEN2_5_0_5B, ModelConfig, get_config  # noqa: F401
from .llama import DecoderLM, StepInput, TPGroup  # noqa: F401
