"""Host-side page bookkeeping: allocator order, compaction plans, request sharding (CPU only)."""

from __future__ import annotations

import random

import numpy as np
import pytest

import cases
import pkv_testlib as lib
from oracle import paged_kv_oracle as oracle
from scheduler import BlockAllocator, KVAllocationError, KVBlockManager, plan_compaction, shard_requests


def test_allocator_follows_reference_pool_order() -> None:
    """Same allocate/release sequence as the reference's PagedKVBlockPool (fixture from its code)."""
    g = lib.golden()
    alloc = None
    results: list[int] = []
    for op, arg in cases.allocator_script():
        if op == "init":
            alloc = BlockAllocator(arg)
        elif op == "allocate":
            results.extend(alloc.allocate(arg))
            results.append(-1)
        else:
            alloc.release(list(arg))
    assert results == g["allocator/results"].tolist()
    assert alloc.free_blocks == g["allocator/free"].tolist()


def test_allocator_rejects_exhaustion_double_release_and_foreign_pages() -> None:
    alloc = BlockAllocator(4)
    pages = alloc.allocate(3)
    with pytest.raises(KVAllocationError):
        alloc.allocate(2)
    alloc.release([pages[0]])
    with pytest.raises(ValueError, match="released twice"):
        alloc.release([pages[0]])
    with pytest.raises(ValueError, match="outside the pool"):
        alloc.release([9])
    with pytest.raises(ValueError, match="not free"):
        alloc.take([pages[1]])


def test_manager_slots_match_the_append_walk() -> None:
    mgr = KVBlockManager(num_pages=32, block_size=4, max_blocks_per_request=8)
    mgr.add_request("a", 5)
    mgr.add_request("b", 0)
    slots_a = mgr.slots_for_append("a", 6)
    slots_b = mgr.slots_for_append("b", 3)
    table_a = mgr.requests["a"].pages
    assert slots_a == oracle.slot_mapping(table_a, 5, 6, 4).tolist()
    assert slots_b == oracle.slot_mapping(mgr.requests["b"].pages, 0, 3, 4).tolist()
    assert mgr.lengths(["a", "b"]) == [11, 3]
    rows = mgr.block_table_rows(["a", "b"])
    assert all(len(r) == 8 for r in rows) and rows[1][1:] == [-1] * 7


def test_manager_rejects_tables_longer_than_max_blocks() -> None:
    mgr = KVBlockManager(num_pages=64, block_size=16, max_blocks_per_request=2)
    with pytest.raises(KVAllocationError):
        mgr.add_request("x", 33)
    mgr.add_request("y", 32)
    with pytest.raises(KVAllocationError):
        mgr.slots_for_append("y", 1)


def test_compaction_plan_is_disjoint_and_packs_live_pages() -> None:
    src, dst = plan_compaction([0, 3, 7, 8, 9], [1, 2, 4, 5, 6])
    assert set(src).isdisjoint(dst)
    assert sorted(set([0, 3, 7, 8, 9]) - set(src) | set(dst)) == [0, 1, 2, 3, 4]
    assert src == [9, 8, 7] and dst == [1, 2, 4]
    assert plan_compaction([0, 1, 2], [3, 4]) == ([], [])
    assert plan_compaction([5, 6], [0, 1, 2, 3, 4], max_moves=1) == ([6], [0])


def test_churn_compaction_preserves_every_request_bit_exactly() -> None:
    """Random finish/arrive churn on a numpy pool: after each compaction (oracle page copy + table remap)
    every request still gathers the tokens it appended."""
    rng = random.Random(5)
    block, pages, heads, dim = 4, 96, 2, 8
    pool = np.zeros((pages, heads, block, dim), dtype=np.float32)
    mgr = KVBlockManager(pages, block, max_blocks_per_request=12)
    content: dict[str, list[np.ndarray]] = {}
    counter = 0
    for step in range(40):
        live = list(mgr.requests)
        for rid in live:
            if rng.random() < 0.15:
                mgr.free_request(rid)
                del content[rid]
        while len(mgr.requests) < 8:
            rid = f"r{counter}"
            counter += 1
            n = rng.randint(1, 30)
            mgr.add_request(rid, 0)
            rows = np.random.default_rng(counter).standard_normal((n, heads, dim)).astype(np.float32)
            oracle.append_slots(pool, np.asarray(mgr.slots_for_append(rid, n)), rows)
            content[rid] = [rows]
        for rid in list(mgr.requests):
            if mgr.requests[rid].length < 40:
                row = np.full((1, heads, dim), step + 0.25, dtype=np.float32)
                oracle.append_slots(pool, np.asarray(mgr.slots_for_append(rid, 1)), row)
                content[rid].append(row)
        if step % 5 == 4:
            before_hw = mgr.high_water()
            src, dst = mgr.compact()
            oracle.copy_pages(pool, src, dst)
            assert set(src).isdisjoint(dst)
            assert mgr.high_water() <= before_hw
            assert mgr.high_water() == len(mgr.live_pages())
        for rid, chunks in content.items():
            expected = np.concatenate(chunks).transpose(1, 0, 2)
            got = oracle.gather_blocks(pool, mgr.requests[rid].pages, mgr.requests[rid].length)
            assert np.array_equal(got, expected), (step, rid)
    assert mgr.copies_planned > 0


def test_shard_requests_balances_tokens_and_covers_every_request() -> None:
    lengths = [8192, 1024, 4096, 3000, 2000, 7000, 1500, 6000, 5000, 2500]
    for world in (1, 2, 4, 8):
        shards = shard_requests(lengths, world)
        assert sorted(i for s in shards for i in s) == list(range(len(lengths)))
        loads = [sum(lengths[i] for i in s) for s in shards]
        assert max(loads) - min(loads) <= max(lengths)
