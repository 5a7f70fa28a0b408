"""Requests and their per-step state.

A request's ``tokens`` are its prompt followed by its outputs. ``num_computed`` counts the leading
tokens whose K/V is in the cache. A step feeds a request either its whole uncomputed prompt
(prefill) or exactly one token at position ``num_computed`` (decode shape). When that position is
the last token, the sampled id is a new output; when it is earlier (after a resume from committed
state), the step is a replay of a position that already has an output, and the sampled id must
equal the recorded one (exact replay).

Reference parity: ``resume_point = min(committed, num_tokens - 1)`` and the one-position-per-step
replay of adapters/vllm/everserve_vllm/resume.py:16-115.
"""

from __future__ import annotations

import enum
import itertools
from dataclasses import dataclass, field

_ids = itertools.count()


class Status(enum.Enum):
    WAITING = "waiting"
    RUNNING = "running"
    FINISHED = "finished"


@dataclass
class SamplingParams:
    """``temperature`` 0 is greedy; otherwise tokens are drawn with ``top_k`` (0: off) and
    ``top_p`` (1: off) from a stream keyed by ``seed`` (default: the request id) and the position,
    so a replayed position draws the same token (everserve_b200.engine.sampling)."""

    max_tokens: int = 16
    eos_id: int | None = None
    ignore_eos: bool = True
    temperature: float = 0.0
    top_k: int = 0
    top_p: float = 1.0
    seed: int | None = None
    logprobs: int | None = None  # None: none; k: each output's log-probability and the k most likely
    stop_ids: tuple = ()  # token ids that end the request (the token is kept as its last output)

    def sampling_key(self, req_id: str) -> tuple[float, int, float, int] | None:
        """What a step needs to sample for this request (None: greedy)."""
        if self.temperature <= 0:
            return None
        from .sampling import default_seed

        seed = self.seed if self.seed is not None else default_seed(req_id)
        return (float(self.temperature), int(self.top_k), float(self.top_p), int(seed) & ((1 << 63) - 1))


@dataclass
class Request:
    prompt: list[int]
    params: SamplingParams = field(default_factory=SamplingParams)
    req_id: str = field(default_factory=lambda: f"req-{next(_ids)}")
    outputs: list[int] = field(default_factory=list)
    status: Status = Status.WAITING
    num_computed: int = 0
    committed: int = 0  # tokens whose K/V the committed-KV store holds
    blocks: list[int] = field(default_factory=list)
    blocks_version: int = 0  # raised whenever the blocks are given back (a new table follows)
    arrival: int = 0
    replay_mismatches: int = 0
    # per output when asked (SamplingParams.logprobs): (log-probability, [(token, log-probability)])
    logprobs: list = field(default_factory=list)

    @property
    def tokens(self) -> list[int]:
        return self.prompt + self.outputs

    def token_at(self, i: int) -> int:
        """tokens[i] without building the list (the decode loop's per-step access)."""
        n = len(self.prompt)
        return self.prompt[i] if i < n else self.outputs[i - n]

    @property
    def num_tokens(self) -> int:
        return len(self.prompt) + len(self.outputs)

    @property
    def finished(self) -> bool:
        return self.status is Status.FINISHED

    def is_prefill(self) -> bool:
        return self.num_computed == 0 and len(self.prompt) > 1

    def done_generating(self) -> bool:
        return self.finish_reason() is not None

    def finish_reason(self) -> str | None:
        """"stop" (an end-of-sequence or stop token), "length" (max_tokens), or None (not done)."""
        if self.outputs:
            last = self.outputs[-1]
            if last in self.params.stop_ids:
                return "stop"
            if not self.params.ignore_eos and self.params.eos_id is not None and last == self.params.eos_id:
                return "stop"
        if len(self.outputs) >= self.params.max_tokens:
            return "length"
        return None

    def resume_point(self) -> int:
        """Where computation restarts after a loss: the committed count, at most the last token."""
        return min(self.committed, self.num_tokens - 1)
