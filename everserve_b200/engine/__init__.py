"""The paged-KV continuous-batching engine."""

from .config import EngineConfig  # noqa: F401
from .engine import Engine, LocalExecutor  # noqa: F401
from .request import Request, SamplingParams  # noqa: F401
