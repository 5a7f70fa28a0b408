"""Seeded sampling that replays exactly: temperature, top-k, top-p, per-request seeds.

Exact replay after a failover needs every sampled token to be a pure function of what the step
sees: the logits row, the request's parameters, its seed and the position it samples at. So the
random numbers here are not drawn from a generator with hidden state: each (seed, position,
vocabulary index) is hashed to a uniform number (a SplitMix64 mix of a Weyl sequence, in int64
arithmetic, which is exact on every device), and the token is the Gumbel-max argmax
``argmax(logits / T + g)`` over the tokens top-k and top-p keep, with ``g = -log(-log(u))``. A
replayed position draws the same numbers, so a spare that re-runs a step samples what the lost
rank sampled. Greedy rows (temperature 0) take the plain argmax; a batch with no sampled row never
enters this module (the decode graphs of greedy batches are unchanged).

All operations are tensor ops with static shapes, so a sampling batch is captured in a CUDA graph
like a greedy one. Ties resolve to the lowest index, as in the argmax kernel.

Reference parity: vLLM's sampler parameters (temperature, top_k, top_p, seed) that the
reference's engine serves; the counter-based draw is this framework's, because exact replay
needs it.
"""

from __future__ import annotations

import hashlib
from dataclasses import dataclass

import torch

# SplitMix64 constants (Steele, Lea, Flood, "Fast splittable pseudorandom number generators",
# OOPSLA 2014), as signed int64
_GOLDEN = 0x9E3779B97F4A7C15 - (1 << 64)
_M1 = 0xBF58476D1CE4E5B9 - (1 << 64)
_M2 = 0x94D049BB133111EB - (1 << 64)
_POS = 0xD1B54A32D192ED03 - (1 << 64)


def default_seed(req_id: str) -> int:
    """A request without a seed draws from a stream keyed by its id (stable across processes)."""
    return int.from_bytes(hashlib.sha256(req_id.encode()).digest()[:8], "little") & ((1 << 63) - 1)


def _shr(x: torch.Tensor, k: int) -> torch.Tensor:
    """Logical right shift of int64 (torch's >> is arithmetic)."""
    return (x >> k) & ((1 << (64 - k)) - 1)


def _mix(x: torch.Tensor) -> torch.Tensor:
    x = (x ^ _shr(x, 30)) * _M1
    x = (x ^ _shr(x, 27)) * _M2
    return x ^ _shr(x, 31)


def uniforms(seed: torch.Tensor, position: torch.Tensor, vocab: int) -> torch.Tensor:
    """[B, vocab] float64 uniforms in (0, 1) for each row's (seed, position)."""
    v = torch.arange(vocab, dtype=torch.int64, device=seed.device)
    base = _mix(seed * _GOLDEN + position * _POS)  # [B]
    x = _mix(base[:, None] + (v[None, :] + 1) * _GOLDEN)
    return (_shr(x, 11).double() + 0.5) * (1.0 / (1 << 53))


@dataclass
class SamplingBatch:
    """Per-row parameters (device tensors of the batch's rows)."""

    temperature: torch.Tensor  # float32 [B]; 0: greedy
    top_k: torch.Tensor  # int64 [B]; 0: off
    top_p: torch.Tensor  # float32 [B]; 1: off
    seed: torch.Tensor  # int64 [B]


def sample(logits: torch.Tensor, positions: torch.Tensor, sb: SamplingBatch) -> torch.Tensor:
    """Tokens [B] (int64) for logits [B, V] sampled at `positions` [B]."""
    x = logits.float()
    B, V = x.shape
    greedy = x.argmax(dim=1)
    temp = sb.temperature.clamp(min=1e-6)
    z = x / temp[:, None]
    # top-k and top-p: one descending sort serves both
    sz, order = torch.sort(z, dim=1, descending=True, stable=True)
    rank = torch.arange(V, device=x.device)[None, :]
    k = torch.where(sb.top_k > 0, sb.top_k.clamp(max=V), torch.full_like(sb.top_k, V))
    keep_sorted = rank < k[:, None]
    probs = torch.softmax(sz, dim=1)
    before = torch.cumsum(probs, dim=1) - probs  # mass of the tokens ranked above
    # the top token is always kept; top_p >= 1 keeps every token (no rounding of the running sum)
    keep_sorted &= (before < sb.top_p[:, None]) | (rank == 0) | (sb.top_p[:, None] >= 1)
    keep = torch.zeros_like(keep_sorted).scatter(1, order, keep_sorted)
    g = -torch.log(-torch.log(uniforms(sb.seed, positions, V)))
    s = torch.where(keep, z.double() + g, torch.full_like(g, float("-inf")))
    drawn = s.argmax(dim=1)
    return torch.where(sb.temperature > 0, drawn, greedy)
