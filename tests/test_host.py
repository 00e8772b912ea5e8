"""Host-side logic on CPU: block tables (bit-exact with the reference's golden random walk
and its known-answer tests), the KV cache bookkeeping, the round bookkeeping helpers, and
the C ABI surface of libspecb200.so."""
from __future__ import annotations

import ctypes
import math
import re

import pytest
import torch

from conftest import ROOT
from cache.kv import KVCache
from cache.paged import BlockAllocator, BlockTable, OutOfBlocks
from spec.loop import SpecStats, finished, record, trim


# ---------------------------------------------------------------- block tables (cache/paged.py)
def test_exhaustion_raises() -> None:
    a = BlockAllocator(3)
    for _ in range(3):
        a.allocate()
    with pytest.raises(OutOfBlocks):
        a.allocate()


def test_double_free_and_foreign_free_raise() -> None:
    a = BlockAllocator(2)
    blk = a.allocate()
    a.free(blk)
    with pytest.raises(ValueError):
        a.free(blk)
    with pytest.raises(ValueError):
        a.free(99)


def test_failed_grow_changes_nothing() -> None:
    a = BlockAllocator(3)
    t = BlockTable()
    t.grow_to(8, a, block_size=4)
    with pytest.raises(OutOfBlocks):
        t.grow_to(13, a, block_size=4)
    assert t.length == 8 and len(t.blocks) == 2 and a.num_free == 1


@pytest.mark.parametrize(("length", "blocks"), [(9, 3), (8, 2), (5, 2), (4, 1), (1, 1), (0, 0)])
def test_shrink_keeps_ceil(length: int, blocks: int) -> None:
    a = BlockAllocator(4)
    t = BlockTable()
    t.grow_to(9, a, block_size=4)
    t.shrink_to(length, a, block_size=4)
    assert len(t.blocks) == blocks and a.num_free == 4 - blocks


def test_slot_arithmetic() -> None:
    t = BlockTable(blocks=[7, 2], length=6)
    assert t.slots(0, 6, block_size=4).tolist() == [28, 29, 30, 31, 8, 9]
    assert t.slots(3, 5, block_size=4).tolist() == [31, 8]


def test_fresh_allocator_hands_out_ascending_ids() -> None:
    a = BlockAllocator(5)
    assert [a.allocate() for _ in range(3)] == [0, 1, 2]
    a.free(1)
    assert a.allocate() == 1  # LIFO: the block freed last comes back first


def _cache(block_size: int, num_blocks: int) -> KVCache:
    return KVCache(n_layers=2, n_kv_heads=2, head_dim=8, num_blocks=num_blocks, block_size=block_size,
                   dtype=torch.float32, device="cpu")


def test_fragmentation_hand_case() -> None:
    cache = _cache(block_size=4, num_blocks=8)
    for s, n in enumerate([5, 8, 1]):
        cache.add(s)
        cache.append([s], [n])
    st = cache.stats()
    assert st.blocks_in_use == 5 and st.slots_allocated == 20 and st.slots_used == 14
    assert st.waste == pytest.approx(0.3)
    assert st.bytes_per_slot == 256 and st.bytes_in_use == 20 * 256


def test_append_slot_maps_match_table_arithmetic() -> None:
    cache = _cache(block_size=4, num_blocks=8)
    cache.add(0)
    cache.add(1)
    cache.append([0, 1], [3, 6])
    sm = cache.append([0, 1], [2, 1])
    assert sm.past.tolist() == [3, 6] and sm.total.tolist() == [5, 7]
    assert sm.write.tolist() == cache.tables[0].slots(3, 5, 4).tolist() + cache.tables[1].slots(6, 7, 4).tolist()
    assert sm.write_index.tolist() == [0, 1, 2]


def test_walk_matches_reference_golden(golden_paged) -> None:
    """Every table's block ids after each of 600 seeded operations equal the reference's."""
    cache = KVCache(n_layers=1, n_kv_heads=1, head_dim=8, num_blocks=golden_paged["num_blocks"],
                    block_size=golden_paged["block_size"], dtype=torch.float32, device="cpu")
    for op, s, arg, snapshot in golden_paged["log"]:
        if op == "add":
            cache.add(s)
        elif op == "append":
            cache.reserve([s], [arg])
        elif op == "append_oob":
            with pytest.raises(OutOfBlocks):
                cache.reserve([s], [arg])
        elif op == "truncate":
            cache.truncate(s, arg)
        else:
            cache.free(s)
        cache.allocator.check()
        assert {str(k): [t.blocks, t.length] for k, t in cache.tables.items()} == snapshot
        for t in cache.tables.values():
            assert len(t.blocks) == math.ceil(t.length / golden_paged["block_size"])


def test_device_tables_layout() -> None:
    cache = _cache(block_size=2, num_blocks=8)
    cache.add(5)
    cache.add(9)
    cache.reserve([5, 9], [3, 5])
    t = cache.device_tables([9, 5])
    assert t.dtype == torch.int32 and t.tolist() == [[2, 3, 4], [0, 1, 0]]


# ---------------------------------------------------------------- round bookkeeping (spec/loop.py)
def test_record_counts_attempts_and_accepts() -> None:
    st = SpecStats(4)
    record(st, 2)
    record(st, 4)
    record(st, 0)
    assert st.drafted == 12 and st.accepted == 6 and st.discarded == 6
    assert st.attempts == [3, 2, 2, 1] and st.accepts == [2, 2, 1, 1]


def test_trim_and_finished() -> None:
    assert trim([1, 2, 3], have=9, max_new_tokens=10, eos_id=None) == [1]
    assert trim([1, 7, 3], have=0, max_new_tokens=10, eos_id=7) == [1, 7]
    assert finished([1, 7], 10, 7) and finished([1] * 10, 10, None) and not finished([1, 2], 10, 7)


# ---------------------------------------------------------------- the C ABI surface
def _declared_symbols() -> list[str]:
    text = (ROOT / "include" / "specb200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(specb200_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol() -> None:
    from specb200 import _ffi

    lib = ctypes.CDLL(str(_ffi.LIB_PATH))
    declared = _declared_symbols()
    assert len(declared) >= 17
    for name in declared:
        assert hasattr(lib, name), name
    assert set(declared) <= set(_ffi.PROTOTYPES), set(declared) - set(_ffi.PROTOTYPES)


def test_host_queries_need_no_gpu() -> None:
    from specb200 import _ffi

    lib = _ffi.lib()
    assert lib.specb200_version() == 10000
    assert lib.specb200_accept_workspace_bytes(64, 4) > 64 * 9 * 16
    assert lib.specb200_attention_workspace_bytes(1, 5, 32, 32, 64, 640) > 0
    assert lib.specb200_linear_workspace_bytes(5, 6144, 2048) > 0


def test_linear_plan_splits_long_k_at_verify_batches() -> None:
    """The workspace a bf16 linear asks for is 4096 B of tile counters plus, when K is split,
    n_tiles x m_tiles x splits x BN x 128 fp32 partials. It shows the plan without a GPU: a long-K
    projection at verify batch sizes keeps 160-token tiles (144 at 288 rows) and splits K 8
    ways, where halving the tile to 32 tokens would make every CTA stream the whole K; prefill
    sizes, short K and the 5-row verify keep their plans."""
    from specb200 import _ffi

    lib = _ffi.lib()
    counters = 4096

    def partials(n_tiles, m_tiles, splits, bn):
        return counters + n_tiles * m_tiles * splits * bn * 128 * 4

    assert lib.specb200_linear_workspace_bytes(320, 2048, 8192) == partials(16, 2, 8, 160)  # B = 64 down
    assert lib.specb200_linear_workspace_bytes(160, 2048, 8192) == partials(16, 1, 8, 160)  # B = 32 down
    assert lib.specb200_linear_workspace_bytes(288, 2048, 8192) == partials(16, 2, 8, 144)  # config 4 down
    assert lib.specb200_linear_workspace_bytes(5, 2048, 8192) == partials(16, 1, 9, 16)  # B = 1 down
    for m, n, k in ((512, 2048, 8192), (320, 6144, 2048), (320, 16384, 2048), (320, 2048, 2048)):
        assert lib.specb200_linear_workspace_bytes(m, n, k) == counters, (m, n, k)  # no K split


def test_host_argument_checks_reject_bad_calls() -> None:
    from specb200 import _ffi

    lib = _ffi.lib()
    assert lib.specb200_accept(None, None, None, None, None, 0, 4, 10, 0, 1.0, None, None, None, None, 0, None) == \
        _ffi.ERR_ARG
    assert lib.specb200_ngram(None, 8, None, 1, 4, 9, None, None, None) == _ffi.ERR_ARG  # max_n > 8
    assert b"max_n" in lib.specb200_last_error()
