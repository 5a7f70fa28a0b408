"""Paged-KV cache layouts and row copies between a cache and staging rows.

A slot is ``block * block_size + offset``. A row is one (slot, kv head) pair: its K and V vectors,
``[2, head_dim]``. Four cache layouts are described by the five element strides the copy kernels
take (block, offset, head, kv, element):

* ``kv_first``      [2, blocks, block_size, heads, d]
* ``blocks_first``  [blocks, 2, block_size, heads, d]
* ``combined``      [blocks, heads, block_size, 2 * d]
* ``heads_blocked`` [blocks, 2, heads, block_size, d]   (this engine's cache: whole (block, head)
  runs are contiguous, which the decode attention kernel streams with bulk copies)

Reference parity: the layouts and strides of core/everserve/state/kvcopy.py:37-140 (the first
three); ``heads_blocked`` is this framework's addition.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

LAYOUTS = ("kv_first", "blocks_first", "combined", "heads_blocked")


@dataclass(frozen=True)
class PagedKV:
    layout: str
    num_blocks: int
    block_size: int
    heads: int
    head_dim: int

    def shape(self) -> tuple[int, ...]:
        B, bs, H, d = self.num_blocks, self.block_size, self.heads, self.head_dim
        return {
            "kv_first": (2, B, bs, H, d),
            "blocks_first": (B, 2, bs, H, d),
            "combined": (B, H, bs, 2 * d),
            "heads_blocked": (B, 2, H, bs, d),
        }[self.layout]

    def strides(self) -> list[int]:
        """Element strides (block, offset, head, kv, element) of a contiguous cache."""
        B, bs, H, d = self.num_blocks, self.block_size, self.heads, self.head_dim
        if self.layout == "kv_first":
            return [bs * H * d, H * d, d, B * bs * H * d, 1]
        if self.layout == "blocks_first":
            return [2 * bs * H * d, H * d, d, bs * H * d, 1]
        if self.layout == "combined":
            return [H * bs * 2 * d, 2 * d, bs * 2 * d, d, 1]
        return [2 * H * bs * d, d, bs * d, H * bs * d, 1]

    def slot(self, block: int, offset: int) -> int:
        return block * self.block_size + offset

    def rows_of_heads(self, cache: torch.Tensor, slots: torch.Tensor, heads: torch.Tensor) -> torch.Tensor:
        """[len(heads), len(slots), 2, d] rows (torch path; padding slots read as zeros)."""
        st = self.strides()
        flat = cache.reshape(-1)
        blk, off = slots.clamp(min=0) // self.block_size, slots.clamp(min=0) % self.block_size
        base = blk * st[0] + off * st[1]
        idx = (base[None, :, None, None] + heads[:, None, None, None] * st[2]
               + torch.arange(2, device=cache.device)[None, None, :, None] * st[3]
               + torch.arange(self.head_dim, device=cache.device)[None, None, None, :])
        rows = flat[idx.reshape(-1)].view(len(heads), len(slots), 2, self.head_dim)
        return rows * (slots >= 0).to(rows.dtype)[None, :, None, None]

    def write_rows(self, cache: torch.Tensor, slots: torch.Tensor, heads: torch.Tensor, rows: torch.Tensor) -> None:
        """Inverse of rows_of_heads: write [len(heads), len(slots), 2, d] rows at the slots."""
        keep = slots >= 0
        if not bool(keep.any()):
            return
        slots, rows = slots[keep], rows[:, keep]
        st = self.strides()
        flat = cache.view(-1)
        blk, off = slots // self.block_size, slots % self.block_size
        base = blk * st[0] + off * st[1]
        idx = (base[None, :, None, None] + heads[:, None, None, None] * st[2]
               + torch.arange(2, device=cache.device)[None, None, :, None] * st[3]
               + torch.arange(self.head_dim, device=cache.device)[None, None, None, :])
        flat[idx.reshape(-1)] = rows.reshape(-1).to(cache.dtype)
