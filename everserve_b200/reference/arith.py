"""Arithmetic of the reference tier: the ops (fp32, HF conventions), the rank-order member sum, and
weight sources that give every unit the same tensor whichever rank loads it.

Reference parity: core/everserve/reference/arith/ops.py:17-73 (rms_norm, inverse frequencies,
rope, member_sum) and arith/sources.py:26-99 (DeterministicSource, SafetensorsSource).
"""

from __future__ import annotations

import hashlib

import torch

from ..ops.ref import cos_sin_table, inverse_frequencies, member_sum, rmsnorm, rope  # noqa: F401


def _seed(seed: int, name: str) -> int:
    return int.from_bytes(hashlib.sha256(f"{seed}:{name}".encode()).digest()[:8], "little") & ((1 << 63) - 1)


class DeterministicSource:
    """Weights from a seed and a name (no files): the same name is the same tensor everywhere."""

    def __init__(self, seed: int = 0, std: float = 0.05):
        self.seed, self.std = seed, std

    def get(self, name: str, shape) -> torch.Tensor:
        g = torch.Generator().manual_seed(_seed(self.seed, name))
        return torch.randn(*shape, generator=g) * self.std


class SafetensorsSource:
    """Weights read from safetensors files (a HF checkpoint directory), sliced by the caller."""

    def __init__(self, directory: str):
        import glob
        import os

        from safetensors import safe_open

        self._files = {}
        for path in sorted(glob.glob(os.path.join(directory, "*.safetensors"))):
            with safe_open(path, framework="pt") as f:
                for k in f.keys():
                    self._files[k] = path
        self._open = safe_open

    def get(self, name: str, shape=None) -> torch.Tensor:
        with self._open(self._files[name], framework="pt") as f:
            t = f.get_tensor(name).float()
        if shape is not None and tuple(t.shape) != tuple(shape):
            raise ValueError(f"{name}: shape {tuple(t.shape)}, expected {tuple(shape)}")
        return t


def row_slice(t: torch.Tensor, i: int, n: int) -> torch.Tensor:
    """Slice i of n equal row blocks."""
    k = t.shape[0] // n
    return t[i * k : (i + 1) * k]


def col_slice(t: torch.Tensor, i: int, n: int) -> torch.Tensor:
    k = t.shape[1] // n
    return t[:, i * k : (i + 1) * k]
