"""Block tables for the paged KV cache, kept on the host.

Same semantics as the reference's cache/paged.py, which the engine must reproduce bit for
bit (block ids are part of the observable state: test_paged's slot arithmetic and random
walk). The kernels never allocate: the round driver grows a table before a forward and
shrinks it after accept-reject, and the forward reads a device copy of the table.

- BlockAllocator (cache/paged.py:11-46): a LIFO free list. It starts as
  [num_blocks-1, ..., 1, 0] and hands out from the end, so a fresh allocator gives 0, 1, 2, ...
  and the block freed last is reused first; a fixed operation sequence always yields the
  same ids.
- BlockTable.grow_to (cache/paged.py:54-62) checks the whole need before taking a block,
  so a failed grow changes nothing (OutOfBlocks); shrink_to (cache/paged.py:64-71) keeps
  ceil(length / block_size) blocks and frees the rest in table order.
- slots (cache/paged.py:73-76): slot = block * block_size + position % block_size.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch


class OutOfBlocks(RuntimeError):
    pass


def _blocks_for(length: int, block_size: int) -> int:
    return -(-length // block_size)


class BlockAllocator:
    def __init__(self, num_blocks: int) -> None:
        self.num_blocks = num_blocks
        self._free: list[int] = list(reversed(range(num_blocks)))
        self._used: set[int] = set()
        self.peak_used = 0

    @property
    def num_free(self) -> int:
        return len(self._free)

    @property
    def num_used(self) -> int:
        return len(self._used)

    def allocate(self) -> int:
        if not self._free:
            raise OutOfBlocks(f"all {self.num_blocks} blocks in use")
        block = self._free.pop()
        self._used.add(block)
        if len(self._used) > self.peak_used:
            self.peak_used = len(self._used)
        return block

    def free(self, block: int) -> None:
        if block not in self._used:
            raise ValueError(f"block {block} is not allocated (double free or foreign id)")
        self._used.discard(block)
        self._free.append(block)

    def check(self) -> None:
        free = set(self._free)
        assert len(free) == len(self._free), "duplicate id in free list"
        assert not free & self._used, "block both free and used"
        assert free | self._used == set(range(self.num_blocks)), "block leaked"


@dataclass
class BlockTable:
    blocks: list[int] = field(default_factory=list)
    length: int = 0

    def grow_to(self, length: int, allocator: BlockAllocator, block_size: int) -> None:
        missing = _blocks_for(length, block_size) - len(self.blocks)
        if missing > allocator.num_free:
            raise OutOfBlocks(f"need {missing} blocks, {allocator.num_free} free")
        self.blocks.extend(allocator.allocate() for _ in range(max(0, missing)))
        self.length = length

    def shrink_to(self, length: int, allocator: BlockAllocator, block_size: int) -> None:
        if length > self.length:
            raise ValueError(f"cannot shrink length {self.length} to {length}")
        keep = _blocks_for(length, block_size)
        for block in self.blocks[keep:]:
            allocator.free(block)
        del self.blocks[keep:]
        self.length = length

    def slots(self, start: int, stop: int, block_size: int) -> torch.Tensor:
        pos = torch.arange(start, stop)
        ids = torch.tensor(self.blocks, dtype=torch.long)
        return ids[pos // block_size] * block_size + pos % block_size


@dataclass(frozen=True)
class FragmentationStats:
    block_size: int
    bytes_per_slot: int
    blocks_in_use: int
    peak_blocks_in_use: int
    slots_used: int

    @property
    def slots_allocated(self) -> int:
        return self.blocks_in_use * self.block_size

    @property
    def waste(self) -> float:
        """Internal fragmentation: the unused tail of each sequence's last block."""
        allocated = self.slots_allocated
        return 0.0 if allocated == 0 else 1.0 - self.slots_used / allocated

    @property
    def bytes_in_use(self) -> int:
        return self.slots_allocated * self.bytes_per_slot

    @property
    def peak_bytes(self) -> int:
        return self.peak_blocks_in_use * self.block_size * self.bytes_per_slot
