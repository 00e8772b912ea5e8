"""Oracle: block allocator and block tables (cache/paged.py:11-76 of the reference).

LIFO free list initialised [num_blocks-1, ..., 0] and popped from the end; grow_to checks the
whole need first (cache/paged.py:54-62); shrink_to keeps ceil(length / block_size) blocks
(cache/paged.py:64-71); slot = block * block_size + position % block_size (cache/paged.py:73-76).
"""
from __future__ import annotations


class OutOfBlocks(RuntimeError):
    pass


class Allocator:
    def __init__(self, num_blocks: int) -> None:
        self.num_blocks = num_blocks
        self.free_list = list(range(num_blocks - 1, -1, -1))
        self.used: set[int] = set()
        self.peak = 0

    def allocate(self) -> int:
        if not self.free_list:
            raise OutOfBlocks("empty")
        b = self.free_list.pop()
        self.used.add(b)
        self.peak = max(self.peak, len(self.used))
        return b

    def release(self, b: int) -> None:
        if b not in self.used:
            raise ValueError(f"block {b} not allocated")
        self.used.remove(b)
        self.free_list.append(b)


class Table:
    def __init__(self) -> None:
        self.blocks: list[int] = []
        self.length = 0

    def grow_to(self, length: int, alloc: Allocator, bs: int) -> None:
        need = -(-length // bs) - len(self.blocks)
        if need > len(alloc.free_list):
            raise OutOfBlocks(f"need {need}")
        for _ in range(need):
            self.blocks.append(alloc.allocate())
        self.length = length

    def shrink_to(self, length: int, alloc: Allocator, bs: int) -> None:
        if length > self.length:
            raise ValueError("grow via shrink")
        keep = -(-length // bs)
        for b in self.blocks[keep:]:
            alloc.release(b)
        self.blocks = self.blocks[:keep]
        self.length = length

    def slots(self, start: int, stop: int, bs: int) -> list[int]:
        return [self.blocks[p // bs] * bs + p % bs for p in range(start, stop)]
