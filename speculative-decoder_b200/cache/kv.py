"""Paged K/V pool for independent sequences (the reference's cache/kv.py:18-127 interface).

The pool keeps the reference's layout, k and v of shape [n_layers, num_blocks * block_size,
n_kv_heads, head_dim]; a slot is one position in the flat pool and each sequence maps its
positions to slots through its BlockTable. On the engine path nothing is copied per step:
the forward's QKV epilogue writes new K/V straight into their slots and the attention
kernel reads blocks in place through a device copy of the block tables
(`device_tables`). Rollback after accept-reject is `truncate`, a table/length edit.

`append`, `write` and `gather` keep the reference's SlotMap interface for callers that use
them directly; the engine's forward uses `reserve` instead, which grows the tables exactly as
`append` does but skips building host-side slot maps.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
from transformers import PretrainedConfig

from cache.paged import BlockAllocator, BlockTable, FragmentationStats


@dataclass(frozen=True)
class SlotMap:
    write: torch.Tensor        # [n_valid] pool slots receiving the new tokens
    write_index: torch.Tensor  # [n_valid] rows of the flattened [B*T] new-token block that are real
    read: torch.Tensor         # [B, S] pool slot of every cached position after the append
    past: torch.Tensor         # [B] cached length before the append
    total: torch.Tensor        # [B] cached length after it


class KVCache:
    def __init__(self, n_layers: int, n_kv_heads: int, head_dim: int, num_blocks: int, block_size: int,
                 dtype: torch.dtype, device: torch.device | str) -> None:
        self.block_size = block_size
        self.device = torch.device(device)
        self.allocator = BlockAllocator(num_blocks)
        shape = (n_layers, num_blocks * block_size, n_kv_heads, head_dim)
        self.k = torch.zeros(shape, dtype=dtype, device=self.device)
        self.v = torch.zeros(shape, dtype=dtype, device=self.device)
        self.tables: dict[int, BlockTable] = {}
        self.bytes_per_slot = 2 * n_layers * n_kv_heads * head_dim * self.k.element_size()

    @classmethod
    def for_model(cls, config: PretrainedConfig, num_blocks: int, block_size: int, dtype: torch.dtype,
                  device: torch.device | str) -> "KVCache":
        head_dim = getattr(config, "head_dim", None) or config.hidden_size // config.num_attention_heads
        return cls(config.num_hidden_layers, config.num_key_value_heads, head_dim, num_blocks, block_size, dtype, device)

    @classmethod
    def contiguous(cls, config: PretrainedConfig, max_batch: int, max_seq_len: int, dtype: torch.dtype,
                   device: torch.device | str) -> "KVCache":
        """One max_seq_len block per sequence: the pre-allocated cache, on the same code."""
        return cls.for_model(config, max_batch, max_seq_len, dtype, device)

    @property
    def num_slots(self) -> int:
        return self.k.shape[1]

    # ---------------------------------------------------------------- sequences
    def add(self, seq_id: int) -> None:
        if seq_id in self.tables:
            raise ValueError(f"sequence {seq_id} already present")
        self.tables[seq_id] = BlockTable()

    def free(self, seq_id: int) -> None:
        self.tables[seq_id].shrink_to(0, self.allocator, self.block_size)
        del self.tables[seq_id]

    def length(self, seq_id: int) -> int:
        return self.tables[seq_id].length

    def truncate(self, seq_id: int, length: int) -> None:
        """Rollback: blocks wholly past `length` go back to the free list; entries past it in
        the kept block are stale but never read (attention stops at the cached length) and
        are overwritten by the next forward before any read."""
        self.tables[seq_id].shrink_to(length, self.allocator, self.block_size)

    def reserve(self, seq_ids: list[int], n_new: list[int]) -> list[int]:
        """Grow each sequence by n_new[b] positions, in order (as append does); returns the
        cached lengths before the growth."""
        past = [self.tables[s].length for s in seq_ids]
        for s, n in zip(seq_ids, n_new):
            table = self.tables[s]
            table.grow_to(table.length + n, self.allocator, self.block_size)
        return past

    def device_tables(self, seq_ids: list[int], width: int | None = None) -> torch.Tensor:
        """[B, width] int32 block ids of each sequence (zero-padded) on the pool's device."""
        rows = [self.tables[s].blocks for s in seq_ids]
        w = max(1, width or max((len(r) for r in rows), default=1))
        host = torch.zeros(len(rows), w, dtype=torch.int32)
        for i, r in enumerate(rows):
            if r:
                host[i, : len(r)] = torch.tensor(r, dtype=torch.int32)
        return host.to(self.device)

    # ---------------------------------------------------------------- reference slot maps
    def append(self, seq_ids: list[int], n_new: list[int]) -> SlotMap:
        """Reserve n_new[b] positions per sequence and return the host-built slot maps of the
        reference (cache/kv.py:79-99). Padded read entries point at slot 0 and must be masked."""
        width = max(n_new)
        past = self.reserve(seq_ids, n_new)
        total = [p + n for p, n in zip(past, n_new)]
        bs = self.block_size
        write = torch.cat([self.tables[s].slots(p, t, bs) for s, p, t in zip(seq_ids, past, total)])
        write_index = torch.cat([b * width + torch.arange(n) for b, n in enumerate(n_new)])
        read = torch.zeros(len(seq_ids), max(total), dtype=torch.long)
        for b, (s, t) in enumerate(zip(seq_ids, total)):
            read[b, :t] = self.tables[s].slots(0, t, bs)
        dev = self.device
        as_dev = lambda x: torch.as_tensor(x, dtype=torch.long).to(dev)  # noqa: E731
        return SlotMap(as_dev(write), as_dev(write_index), as_dev(read), as_dev(past), as_dev(total))

    def write(self, layer: int, slots: SlotMap, k: torch.Tensor, v: torch.Tensor) -> None:
        """k, v: [B, H_kv, T, d] for the tokens passed to append, right-padded to T."""
        b, h, t, d = k.shape
        rows = slots.write_index
        self.k[layer][slots.write] = k.transpose(1, 2).reshape(b * t, h, d)[rows]
        self.v[layer][slots.write] = v.transpose(1, 2).reshape(b * t, h, d)[rows]

    def gather(self, layer: int, slots: SlotMap) -> tuple[torch.Tensor, torch.Tensor]:
        """[B, H_kv, S, d] copies of every cached position (the engine never calls this)."""
        return self.k[layer][slots.read].transpose(1, 2), self.v[layer][slots.read].transpose(1, 2)

    def stats(self) -> FragmentationStats:
        return FragmentationStats(
            block_size=self.block_size,
            bytes_per_slot=self.bytes_per_slot,
            blocks_in_use=self.allocator.num_used,
            peak_blocks_in_use=self.allocator.peak_used,
            slots_used=sum(t.length for t in self.tables.values()),
        )
