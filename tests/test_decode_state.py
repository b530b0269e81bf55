"""decode_state on shared device pools: host-side behaviour on CPU, data path on the GPU.

The GPU tests follow the reference's own decode_state tests (tests/unit/test_decode_state.py:33-439 in
the reference project) -- append equals concatenation across blocks, prefill then single steps,
release reuses blocks, reordered tables gather in logical order, batched tables pad with -1 -- with
KV heads stored once and all requests of a layer in one pool.
"""

from __future__ import annotations

from types import SimpleNamespace

import pytest
import torch

from decode_state import (
    DEFAULT_KV_BLOCK_SIZE,
    DecodeState,
    FullAttentionCache,
    FullAttentionCacheStats,
    LinearAttentionCache,
    PagedKVBlockPool,
    batch_kv_tensors,
    batch_page_tables,
)

DEVICE = "cuda:0"


def _kv(step: int, *, heads: int = 2, seq: int = 1, head_dim: int = 4, device: str = DEVICE):
    base = float(step * 1000)
    count = heads * seq * head_dim
    key = (base + torch.arange(count, dtype=torch.float32)).reshape(1, heads, seq, head_dim)
    value = (base + 0.5 + torch.arange(count, dtype=torch.float32)).reshape(1, heads, seq, head_dim)
    return key.to(device), value.to(device)


def _mapping(types):
    return SimpleNamespace(layers=tuple(SimpleNamespace(index=i, layer_type=t) for i, t in enumerate(types)))


# ---- CPU: host-side behaviour ------------------------------------------------------------------------------
def test_stats_keep_the_reference_field_names() -> None:
    assert list(FullAttentionCacheStats.__dataclass_fields__) == [
        "block_size", "valid_tokens", "capacity_tokens", "logical_blocks", "allocated_blocks", "free_blocks",
        "append_calls", "appended_tokens", "growth_events", "release_calls", "released_blocks",
        "contiguous_view_calls", "gather_view_calls", "gather_copied_tokens", "page_table_tensor_calls",
        "page_metadata_calls", "batched_page_table_calls", "page_table_entries_total", "non_contiguous",
        "estimated_key_bytes", "estimated_value_bytes", "estimated_total_bytes",
    ]


def test_decode_state_empty_threads_hint_block_size_and_pools() -> None:
    state = DecodeState.empty(_mapping(("full_attention", "linear_attention", "full_attention")), None,
                              max_seq_len=16, kv_block_size=4)
    full = [layer for layer in state.layers if isinstance(layer, FullAttentionCache)]
    assert len(full) == 2 and isinstance(state.layers[1], LinearAttentionCache)
    assert all(c.capacity_hint == 16 and c.block_size == 4 for c in full)
    assert full[0].key_blocks is None  # private pools are created lazily
    assert DecodeState.empty(_mapping(("full_attention",))).layers[0].block_size == DEFAULT_KV_BLOCK_SIZE


def test_slot_mapping_walks_the_table() -> None:
    cache = FullAttentionCache(block_size=4)
    cache.block_table = [7, 2, 9]
    assert cache.slot_mapping(3, 6) == [31, 8, 9, 10, 11, 36]


def test_cpu_tensors_are_rejected_not_emulated() -> None:
    cache = FullAttentionCache(capacity_hint=4, block_size=2)
    key, value = _kv(0, device="cpu")
    with pytest.raises(RuntimeError, match="must be CUDA"):
        cache.append_blocks(key, value)


# ---- GPU: data path --------------------------------------------------------------------------------------------
@pytest.mark.gpu
def test_append_returns_tensors_equal_to_manual_concat() -> None:
    cache = FullAttentionCache(block_size=2)
    keys, values = [], []
    for step in range(5):
        key, value = _kv(step)
        keys.append(key)
        values.append(value)
        out_key, out_value = cache.append(key, value)
        assert torch.equal(out_key, torch.cat(keys, dim=2))
        assert torch.equal(out_value, torch.cat(values, dim=2))


@pytest.mark.gpu
def test_prefill_chunk_then_single_steps_across_blocks() -> None:
    cache = FullAttentionCache(block_size=2)
    k0, v0 = _kv(0, seq=3)
    keys, values = [k0], [v0]
    cache.append(k0, v0)
    for step in range(1, 4):
        k, v = _kv(step)
        keys.append(k)
        values.append(v)
        out_key, out_value = cache.append(k, v)
    assert torch.equal(out_key, torch.cat(keys, dim=2)) and torch.equal(out_value, torch.cat(values, dim=2))
    assert cache.block_table == [0, 1, 2, 3]
    assert cache.capacity == 8


@pytest.mark.gpu
def test_release_reuses_blocks_of_a_shared_pool() -> None:
    pool = PagedKVBlockPool.shared(8, 2, 4, block_size=2, dtype=torch.float32, device=DEVICE)
    a = FullAttentionCache(capacity_hint=4, block_size=2, pool=pool)
    b = FullAttentionCache(capacity_hint=4, block_size=2, pool=pool)
    a.append(*_kv(0, seq=3))
    b.append(*_kv(1, seq=3))
    assert a.block_table == [0, 1] and b.block_table == [2, 3]
    released = list(a.block_table)
    a.release()
    assert a.length == 0 and a.block_table == []
    c = FullAttentionCache(capacity_hint=4, block_size=2, pool=pool)
    out_key, _ = c.append(*_kv(2, seq=2))
    assert c.block_table == released
    assert torch.equal(out_key, _kv(2, seq=2)[0])
    assert torch.equal(b.as_tensors()[0], _kv(1, seq=3)[0])


@pytest.mark.gpu
def test_reordered_table_gathers_in_logical_order() -> None:
    pool = PagedKVBlockPool.shared(3, 2, 4, block_size=2, dtype=torch.float32, device=DEVICE)
    cache = FullAttentionCache(capacity_hint=6, block_size=2, pool=pool)
    parts = [_kv(i, seq=2) for i in range(3)]
    for key, value in parts:
        cache.append(key, value)
    cache.block_table = [2, 0, 1]
    for page, (key, value) in zip((2, 0, 1), parts):  # a page is (kv_heads, block_size, head_dim)
        pool.key_blocks[page] = key[0]
        pool.value_blocks[page] = value[0]
    out_key, out_value = cache.as_tensors()
    assert torch.equal(out_key, torch.cat([p[0] for p in parts], dim=2))
    assert torch.equal(out_value, torch.cat([p[1] for p in parts], dim=2))
    assert cache.stats().non_contiguous is True


@pytest.mark.gpu
def test_private_pool_growth_preserves_contents() -> None:
    cache = FullAttentionCache(capacity_hint=2, block_size=2)
    keys = []
    for step in range(6):
        key, value = _kv(step)
        keys.append(key)
        out_key, _ = cache.append(key, value)
    assert torch.equal(out_key, torch.cat(keys, dim=2))
    assert cache.pool.growth_events >= 1 and cache.capacity >= cache.length


@pytest.mark.gpu
def test_batch_page_tables_and_kv_tensors_pad_and_mask() -> None:
    pool = PagedKVBlockPool.shared(16, 2, 4, block_size=2, dtype=torch.float32, device=DEVICE)
    a = FullAttentionCache(block_size=2, pool=pool)
    b = FullAttentionCache(block_size=2, pool=pool)
    a.append_blocks(*_kv(0, seq=3))
    b.append_blocks(*_kv(1, seq=5))
    meta = batch_page_tables([a, b])
    assert meta.block_tables[0].tolist()[len(a.block_table):] == [-1] * (meta.max_blocks - len(a.block_table))
    assert meta.sequence_lengths.tolist() == [3, 5]
    assert meta.valid_mask.tolist() == [[True] * 3 + [False] * 2, [True] * 5]
    keys, values, mask = batch_kv_tensors([a, b])
    assert keys.shape == (2, 2, 5, 4)
    assert torch.equal(keys[0:1, :, :3], _kv(0, seq=3)[0]) and bool((keys[0, :, 3:] == 0).all())
    assert torch.equal(values[1:2], _kv(1, seq=5)[1])
    # caches with private pools are batched too (the reference's per-request pools); a cache without
    # storage is not
    with pytest.raises(ValueError, match="allocated block storage"):
        batch_page_tables([a, FullAttentionCache(block_size=2)])
    c = FullAttentionCache(block_size=2)
    c.append_blocks(*_kv(2, seq=4))
    meta = batch_page_tables([a, c])
    assert meta.key_blocks[0] is pool.key_blocks and meta.key_blocks[1] is c.pool.key_blocks
    keys, _, _ = batch_kv_tensors([a, c])
    assert torch.equal(keys[1:2, :, :4], _kv(2, seq=4)[0]) and torch.equal(keys[0:1, :, :3], _kv(0, seq=3)[0])


@pytest.mark.gpu
def test_decode_over_caches_matches_dense_reference() -> None:
    from tp_runtime import paged_decode_caches

    torch.manual_seed(5)
    pool = PagedKVBlockPool.shared(64, 2, 64, block_size=16, dtype=torch.float16, device=DEVICE)
    caches, dense = [], []
    for n in (5, 40, 100):
        c = FullAttentionCache(block_size=16, pool=pool)
        k = torch.randn((1, 2, n, 64), device=DEVICE, dtype=torch.float16)
        v = torch.randn((1, 2, n, 64), device=DEVICE, dtype=torch.float16)
        c.append_blocks(k, v)
        caches.append(c)
        dense.append((k, v))
    query = torch.randn((3, 16, 1, 64), device=DEVICE, dtype=torch.float16)
    out = paged_decode_caches(query, caches)
    for r, (k, v) in enumerate(dense):
        kk = k.float().repeat_interleave(8, dim=1)
        vv = v.float().repeat_interleave(8, dim=1)
        probs = torch.softmax(query[r : r + 1].float() @ kk.transpose(2, 3) * 64 ** -0.5, dim=-1)
        torch.testing.assert_close(out[r : r + 1].float(), probs @ vv, atol=2e-3, rtol=1e-2)


@pytest.mark.gpu
def test_kv_stats_aggregate_a_decode_state() -> None:
    state = DecodeState.empty(_mapping(("full_attention", "linear_attention", "full_attention")), None,
                              max_seq_len=4, kv_block_size=2)
    for layer in state.layers:
        if isinstance(layer, FullAttentionCache):
            layer.append(*_kv(layer.block_size, seq=2))
    stats = state.kv_stats()
    assert stats.full_attention_layers == 2 and stats.block_size == 2
    assert stats.valid_tokens_total == 4 and stats.capacity_tokens_total == 8
    assert stats.append_calls_total == 2 and stats.estimated_total_bytes > 0
    state.release()
    assert all(layer.length == 0 for layer in state.layers if isinstance(layer, FullAttentionCache))
