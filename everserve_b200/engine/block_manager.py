"""Paged-KV block allocation.

Blocks are fixed-size runs of ``block_size`` token slots. A request owns a list of block ids (its
block table); token position p lives at slot ``blocks[p // block_size] * block_size + p %
block_size``. Free blocks are handed out lowest id first, so two engines that see the same request
sequence lay their caches out identically (a spare's restore writes to the slots the lost rank
used).
"""

from __future__ import annotations

import heapq


class BlockManager:
    def __init__(self, num_blocks: int, block_size: int):
        assert num_blocks > 0 and block_size > 0
        self.num_blocks = num_blocks
        self.block_size = block_size
        self._free = list(range(num_blocks))
        heapq.heapify(self._free)

    @property
    def free_blocks(self) -> int:
        return len(self._free)

    def blocks_for(self, num_tokens: int) -> int:
        return (num_tokens + self.block_size - 1) // self.block_size

    def can_grow(self, blocks: list[int], num_tokens: int) -> bool:
        return self.blocks_for(num_tokens) - len(blocks) <= len(self._free)

    def grow(self, blocks: list[int], num_tokens: int) -> None:
        """Extend a block table in place to cover num_tokens positions."""
        need = self.blocks_for(num_tokens) - len(blocks)
        if need > len(self._free):
            raise MemoryError(f"need {need} KV blocks, {len(self._free)} free")
        for _ in range(max(0, need)):
            blocks.append(heapq.heappop(self._free))

    def free(self, blocks: list[int]) -> None:
        for b in blocks:
            heapq.heappush(self._free, b)
        blocks.clear()

    def take(self, ids: list[int]) -> None:
        """Mark specific blocks used (a restore that must reproduce another engine's layout)."""
        s = set(ids)
        self._free = [b for b in self._free if b not in s]
        heapq.heapify(self._free)

    def slot(self, blocks: list[int], pos: int) -> int:
        return blocks[pos // self.block_size] * self.block_size + pos % self.block_size
