"""Full-attention KV state on shared device page pools (the reference's decode_state, B200 layout).

Same public names as the reference module (src/decode_state.py): PagedKVBlockPool, FullAttentionCache,
FullAttentionPageTable, BatchedFullAttentionPageTables, FullAttentionCacheStats, KVCacheStats,
LinearAttentionCache, DecodeState, batch_kv_tensors, batch_page_tables, DEFAULT_KV_BLOCK_SIZE.
What changes underneath:

  * a pool holds one layer's pages for MANY requests, laid out (num_pages, num_kv_heads, block_size,
    head_dim) with KV heads not repeated; it is sized once (a fixed HBM reservation) and hands out
    page ids from a sorted free list (scheduler.BlockAllocator). A cache created without a pool gets
    a private one, which grows like the reference's (src/decode_state.py:47-70) when needed;
  * append_blocks writes the new tokens with ONE launch (kv_append_positions) instead of a Python
    loop of slice copies: the kernel walks the block table itself (the reference's physical_block /
    block_offset walk, src/decode_state.py:278-284), reading a device copy of the table that is
    re-uploaded only when the table changes (growth, release, a compaction remap) -- no host-built
    slot list and no host->device copy per call;
  * batch_page_tables stages the padded tables of all rows in pinned memory and moves them with one
    asynchronous copy; caches with private pools are served too (per-request pools, as the
    reference's batched kernel takes them);
  * as_tensors / batch_kv_tensors gather through the block table on the device (kv_gather) for
    callers that still want dense K/V; attention never needs them (paged_decode walks the tables);
  * tables are int64 on request (page_table_tensor, as the reference) and int32 for the runner.

Inputs keep the reference's head-major layout (batch, heads, seq, head_dim) with batch 1 per cache,
where `heads` are the KV heads this rank stores.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Sequence

import paged_kv_ops as ops
from scheduler import BlockAllocator

DEFAULT_KV_BLOCK_SIZE = 16


class PagedKVBlockPool:
    """One layer's page pool: K and V (num_pages, num_kv_heads, block_size, head_dim) + free list.

    Created sized (shared pool) or lazily on the first allocation of a private cache. allocate() and
    release() follow the reference pool (src/decode_state.py:72-84): lowest free ids first, released
    ids return to the sorted free list.
    """

    def __init__(self, block_size: int, *, num_pages: int = 0, num_kv_heads: int = 0, head_dim: int = 0,
                 dtype: Any = None, device: Any = None, growable: bool = False) -> None:
        if block_size <= 0:
            raise ValueError("block_size must be positive")
        self.block_size = block_size
        self.growable = growable
        self.key_blocks: Any | None = None
        self.value_blocks: Any | None = None
        self.allocator: BlockAllocator | None = None
        self.growth_events = 0
        if num_pages > 0:
            self._create(num_pages, num_kv_heads, head_dim, dtype, device)

    @classmethod
    def shared(cls, num_pages: int, num_kv_heads: int, head_dim: int, *, block_size: int = DEFAULT_KV_BLOCK_SIZE,
               dtype: Any, device: Any) -> PagedKVBlockPool:
        return cls(block_size, num_pages=num_pages, num_kv_heads=num_kv_heads, head_dim=head_dim, dtype=dtype,
                   device=device, growable=False)

    def _create(self, num_pages: int, num_kv_heads: int, head_dim: int, dtype: Any, device: Any) -> None:
        import torch

        shape = (num_pages, num_kv_heads, self.block_size, head_dim)
        self.key_blocks = torch.empty(shape, dtype=dtype, device=device)
        self.value_blocks = torch.empty(shape, dtype=dtype, device=device)
        self.allocator = BlockAllocator(num_pages)

    @property
    def block_count(self) -> int:
        return 0 if self.key_blocks is None else self.key_blocks.shape[0]

    @property
    def free_blocks(self) -> list[int]:
        return [] if self.allocator is None else self.allocator.free_blocks

    def ensure_initialized(self, key: Any, value: Any, blocks: int) -> None:
        """Creates the pool for `blocks` pages shaped after key (1, kv_heads, seq, head_dim)."""
        if blocks <= 0 or self.key_blocks is not None:
            return
        _batch, heads, _seq, head_dim = key.shape
        self._create(blocks, heads, head_dim, key.dtype, key.device)

    def allocate(self, count: int, key: Any = None, value: Any = None) -> list[int]:
        if self.key_blocks is None:
            if key is None:
                raise RuntimeError("pool is not initialised")
            self.ensure_initialized(key, value, max(count, 1))
        assert self.allocator is not None
        if count > self.allocator.num_free:
            if not self.growable:
                raise RuntimeError(f"KV pool exhausted: need {count} pages, {self.allocator.num_free} free")
            self._grow(count - self.allocator.num_free)
        return self.allocator.allocate(count)

    def release(self, blocks: list[int]) -> None:
        if blocks and self.allocator is not None:
            self.allocator.release(blocks)

    def _grow(self, blocks: int) -> None:
        """Private-pool growth: a larger pool with the old pages copied to the same ids."""
        import torch

        old = self.block_count
        new = max(old + blocks, 2 * old)
        grown_k = torch.empty((new, *self.key_blocks.shape[1:]), dtype=self.key_blocks.dtype,
                              device=self.key_blocks.device)
        grown_v = torch.empty_like(grown_k)
        grown_k[:old].copy_(self.key_blocks)
        grown_v[:old].copy_(self.value_blocks)
        used = [p for p in range(old) if p not in set(self.allocator.free_blocks)]
        self.key_blocks, self.value_blocks = grown_k, grown_v
        allocator = BlockAllocator(new)
        allocator.take(used)
        self.allocator = allocator
        self.growth_events += 1


@dataclass(frozen=True)
class FullAttentionPageTable:
    block_table: Any
    sequence_length: int
    block_size: int
    logical_blocks: int
    capacity_tokens: int
    key_blocks: Any
    value_blocks: Any


@dataclass(frozen=True)
class BatchedFullAttentionPageTables:
    block_tables: Any
    sequence_lengths: Any
    valid_mask: Any
    block_size: int
    max_blocks: int
    max_sequence_length: int
    key_blocks: tuple[Any, ...]
    value_blocks: tuple[Any, ...]


_CACHE_STAT_FIELDS = (
    "block_size", "valid_tokens", "capacity_tokens", "logical_blocks", "allocated_blocks", "free_blocks",
    "append_calls", "appended_tokens", "growth_events", "release_calls", "released_blocks",
    "contiguous_view_calls", "gather_view_calls", "gather_copied_tokens", "page_table_tensor_calls",
    "page_metadata_calls", "batched_page_table_calls", "page_table_entries_total", "non_contiguous",
    "estimated_key_bytes", "estimated_value_bytes", "estimated_total_bytes",
)


@dataclass(frozen=True)
class FullAttentionCacheStats:
    block_size: int
    valid_tokens: int
    capacity_tokens: int
    logical_blocks: int
    allocated_blocks: int
    free_blocks: int
    append_calls: int
    appended_tokens: int
    growth_events: int
    release_calls: int
    released_blocks: int
    contiguous_view_calls: int
    gather_view_calls: int
    gather_copied_tokens: int
    page_table_tensor_calls: int
    page_metadata_calls: int
    batched_page_table_calls: int
    page_table_entries_total: int
    non_contiguous: bool
    estimated_key_bytes: int
    estimated_value_bytes: int
    estimated_total_bytes: int

    def to_dict(self) -> dict[str, int | bool]:
        return {name: getattr(self, name) for name in _CACHE_STAT_FIELDS}


@dataclass(frozen=True)
class KVCacheStats:
    full_attention_layers: int
    block_size: int | None
    valid_tokens_total: int
    capacity_tokens_total: int
    logical_blocks_total: int
    allocated_blocks_total: int
    free_blocks_total: int
    append_calls_total: int
    appended_tokens_total: int
    growth_events_total: int
    release_calls_total: int
    released_blocks_total: int
    contiguous_view_calls_total: int
    gather_view_calls_total: int
    gather_copied_tokens_total: int
    page_table_tensor_calls_total: int
    page_metadata_calls_total: int
    batched_page_table_calls_total: int
    page_table_entries_total: int
    non_contiguous_layers: int
    estimated_total_bytes: int
    max_valid_tokens: int
    max_capacity_tokens: int

    def to_dict(self) -> dict[str, int | None]:
        return dict(vars(self))


@dataclass
class FullAttentionCache:
    """One request's pages of one full-attention layer.

    `append` / `append_blocks` take post-RoPE K/V (1, kv_heads, seq, head_dim); `block_table` maps
    logical blocks to pages of `pool`, which may be shared with other requests.
    """

    capacity_hint: int | None = None
    block_size: int = DEFAULT_KV_BLOCK_SIZE
    pool: PagedKVBlockPool | None = None
    valid: int = 0
    block_table: list[int] = field(default_factory=list)
    append_calls: int = 0
    appended_tokens: int = 0
    growth_events: int = 0
    release_calls: int = 0
    released_blocks: int = 0
    contiguous_view_calls: int = 0
    gather_view_calls: int = 0
    gather_copied_tokens: int = 0
    page_table_tensor_calls: int = 0
    page_metadata_calls: int = 0
    batched_page_table_calls: int = 0
    page_table_entries_total: int = 0
    _table_device: Any = field(default=None, repr=False, compare=False)
    _table_uploaded: list[int] = field(default_factory=list, repr=False, compare=False)

    def __post_init__(self) -> None:
        if self.block_size <= 0:
            raise ValueError("block_size must be positive")
        if self.pool is None:
            self.pool = PagedKVBlockPool(self.block_size, growable=True)
        elif self.pool.block_size != self.block_size:
            raise ValueError("pool block_size differs from the cache's")

    @property
    def key_blocks(self) -> Any | None:
        return self.pool.key_blocks

    @property
    def value_blocks(self) -> Any | None:
        return self.pool.value_blocks

    @property
    def length(self) -> int:
        return self.valid

    @property
    def capacity(self) -> int:
        return len(self.block_table) * self.block_size

    def append(self, key: Any, value: Any) -> tuple[Any, Any]:
        self.append_blocks(key, value)
        return self.as_tensors()

    def slot_mapping(self, start: int, count: int) -> list[int]:
        """Slots of logical positions [start, start+count): page * block_size + offset."""
        bs = self.block_size
        return [self.block_table[p // bs] * bs + p % bs for p in range(start, start + count)]

    def device_block_table(self) -> Any:
        """The block table as an int64 tensor on the pool's device, uploaded again only when the table
        changed since the last upload (growth, release or a compaction remap of `block_table`)."""
        import torch

        device = self.pool.key_blocks.device
        if (self._table_device is None or self._table_device.device != device
                or self._table_uploaded != self.block_table):
            self._table_device = torch.tensor(self.block_table, dtype=torch.int64, device=device)
            self._table_uploaded = list(self.block_table)
        return self._table_device

    def append_blocks(self, key: Any, value: Any) -> None:
        """Writes new K/V (1, kv_heads, seq, head_dim) into this request's pages with one launch that
        reads the device copy of the block table."""
        batch, _heads, seq, _head_dim = key.shape
        if batch != 1:
            raise ValueError("FullAttentionCache holds one request (batch 1)")
        self.append_calls += 1
        self.appended_tokens += int(seq)
        needed = self.valid + seq
        self._ensure_logical_capacity(needed, key, value)
        if seq:
            ops.kv_append_positions(key[0].transpose(0, 1), value[0].transpose(0, 1), self.device_block_table(),
                                    self.valid, self.pool.key_blocks, self.pool.value_blocks)
        self.valid = needed

    def as_tensors(self) -> tuple[Any, Any]:
        """Dense (1, kv_heads, valid, head_dim) K and V gathered through the table."""
        import torch

        if self.valid == 0:
            raise ValueError("FullAttentionCache has no valid tokens")
        self.gather_view_calls += 1
        self.gather_copied_tokens += self.valid
        table = torch.tensor([self.block_table], dtype=torch.int64, device=self.pool.key_blocks.device)
        lens = torch.tensor([self.valid], dtype=torch.int64, device=self.pool.key_blocks.device)
        return ops.kv_gather(self.pool.key_blocks, self.pool.value_blocks, table, lens, self.valid)

    def page_table_tensor(self, *, device: Any | None = None) -> Any:
        import torch

        if device is None and self.pool.key_blocks is not None:
            device = self.pool.key_blocks.device
        self.page_table_tensor_calls += 1
        return torch.tensor(self.block_table, dtype=torch.long, device=device)

    def page_metadata(self) -> FullAttentionPageTable:
        """The request's page table for the decode kernels (src/decode_state.py:314-328); the table is
        the cached device copy (device_block_table), not a fresh upload per call."""
        if self.pool.key_blocks is None:
            raise ValueError("FullAttentionCache page metadata requires allocated block storage")
        self.page_table_tensor_calls += 1
        table = self.device_block_table()
        self.page_metadata_calls += 1
        self.page_table_entries_total += len(self.block_table)
        return FullAttentionPageTable(table, self.valid, self.block_size, len(self.block_table), self.capacity,
                                      self.pool.key_blocks, self.pool.value_blocks)

    def release(self) -> None:
        self.release_calls += 1
        self.released_blocks += len(self.block_table)
        self.pool.release(self.block_table)
        self.block_table = []
        self.valid = 0

    def stats(self) -> FullAttentionCacheStats:
        key_bytes = _tensor_nbytes(self.pool.key_blocks)
        value_bytes = _tensor_nbytes(self.pool.value_blocks)
        return FullAttentionCacheStats(
            block_size=self.block_size,
            valid_tokens=self.valid,
            capacity_tokens=self.capacity,
            logical_blocks=len(self.block_table),
            allocated_blocks=self.pool.block_count,
            free_blocks=len(self.pool.free_blocks),
            append_calls=self.append_calls,
            appended_tokens=self.appended_tokens,
            growth_events=self.growth_events,
            release_calls=self.release_calls,
            released_blocks=self.released_blocks,
            contiguous_view_calls=self.contiguous_view_calls,
            gather_view_calls=self.gather_view_calls,
            gather_copied_tokens=self.gather_copied_tokens,
            page_table_tensor_calls=self.page_table_tensor_calls,
            page_metadata_calls=self.page_metadata_calls,
            batched_page_table_calls=self.batched_page_table_calls,
            page_table_entries_total=self.page_table_entries_total,
            non_contiguous=not self._is_contiguous_table(),
            estimated_key_bytes=key_bytes,
            estimated_value_bytes=value_bytes,
            estimated_total_bytes=key_bytes + value_bytes,
        )

    def _ensure_logical_capacity(self, needed: int, key: Any, value: Any) -> None:
        """Same growth rule as the reference (src/decode_state.py:365-374): at least `needed`, the hint,
        and double the current capacity."""
        if needed <= self.capacity:
            return
        target_tokens = max(needed, self.capacity_hint or 0, max(self.block_size, self.capacity * 2))
        target_blocks = -(-target_tokens // self.block_size)
        missing = target_blocks - len(self.block_table)
        if missing <= 0:
            return
        self.growth_events += 1
        self.block_table.extend(self.pool.allocate(missing, key, value))

    def _is_contiguous_table(self) -> bool:
        if not self.block_table:
            return True
        start = self.block_table[0]
        return self.block_table == list(range(start, start + len(self.block_table)))


def _tensor_nbytes(tensor: Any | None) -> int:
    return 0 if tensor is None else int(tensor.numel() * tensor.element_size())


@dataclass
class LinearAttentionCache:
    """Recurrent + conv state of a gated-delta layer (holds no pages; unchanged from the reference)."""

    state: Any | None = None
    conv_tail: Any | None = None


LayerCache = FullAttentionCache | LinearAttentionCache


@dataclass
class DecodeState:
    """Per-layer caches of one request plus the number of tokens consumed."""

    layers: list[LayerCache]
    position_offset: int = 0

    @classmethod
    def empty(cls, mapping: Any, config: Any = None, max_seq_len: int | None = None, *,
              kv_block_size: int = DEFAULT_KV_BLOCK_SIZE, pools: Sequence[PagedKVBlockPool] | None = None
              ) -> DecodeState:
        """One cache per layer of `mapping.layers` (full-attention layers get a FullAttentionCache on
        pools[i] -- the i-th full-attention layer's shared pool -- or a private pool)."""
        del config
        layers: list[LayerCache] = []
        full_index = 0
        for layer in mapping.layers:
            if layer.layer_type == "full_attention":
                pool = None if pools is None else pools[full_index]
                layers.append(FullAttentionCache(capacity_hint=max_seq_len, block_size=kv_block_size, pool=pool))
                full_index += 1
            else:
                layers.append(LinearAttentionCache())
        return cls(layers=layers, position_offset=0)

    def advance(self, tokens: int) -> None:
        self.position_offset += tokens

    def release(self) -> None:
        for layer in self.layers:
            if isinstance(layer, FullAttentionCache):
                layer.release()

    def kv_stats(self) -> KVCacheStats:
        stats = [layer.stats() for layer in self.layers if isinstance(layer, FullAttentionCache)]
        sizes = {s.block_size for s in stats}
        # a shared pool is counted once
        pools = {id(layer.pool): layer for layer in self.layers if isinstance(layer, FullAttentionCache)}
        return KVCacheStats(
            full_attention_layers=len(stats),
            block_size=next(iter(sizes)) if len(sizes) == 1 else None,
            valid_tokens_total=sum(s.valid_tokens for s in stats),
            capacity_tokens_total=sum(s.capacity_tokens for s in stats),
            logical_blocks_total=sum(s.logical_blocks for s in stats),
            allocated_blocks_total=sum(s.allocated_blocks for s in stats),
            free_blocks_total=sum(s.free_blocks for s in stats),
            append_calls_total=sum(s.append_calls for s in stats),
            appended_tokens_total=sum(s.appended_tokens for s in stats),
            growth_events_total=sum(s.growth_events for s in stats),
            release_calls_total=sum(s.release_calls for s in stats),
            released_blocks_total=sum(s.released_blocks for s in stats),
            contiguous_view_calls_total=sum(s.contiguous_view_calls for s in stats),
            gather_view_calls_total=sum(s.gather_view_calls for s in stats),
            gather_copied_tokens_total=sum(s.gather_copied_tokens for s in stats),
            page_table_tensor_calls_total=sum(s.page_table_tensor_calls for s in stats),
            page_metadata_calls_total=sum(s.page_metadata_calls for s in stats),
            batched_page_table_calls_total=sum(s.batched_page_table_calls for s in stats),
            page_table_entries_total=sum(s.page_table_entries_total for s in stats),
            non_contiguous_layers=sum(1 for s in stats if s.non_contiguous),
            estimated_total_bytes=sum(_tensor_nbytes(c.pool.key_blocks) + _tensor_nbytes(c.pool.value_blocks)
                                      for c in pools.values()),
            max_valid_tokens=max((s.valid_tokens for s in stats), default=0),
            max_capacity_tokens=max((s.capacity_tokens for s in stats), default=0),
        )


def batch_page_tables(caches: Sequence[FullAttentionCache], *, index_dtype: Any = None
                      ) -> BatchedFullAttentionPageTables:
    """-1 padded (B, max_blocks) tables, lengths and valid mask of a batch of caches
    (src/decode_state.py:545-603 semantics): key_blocks/value_blocks hold each row's pool -- the same
    tensor for every row when the caches share one pool. The rows are staged in pinned host memory
    and reach the device with one asynchronous copy; the valid mask is computed on the device."""
    import torch

    if not caches:
        raise ValueError("batch_page_tables requires at least one cache")
    if len({c.block_size for c in caches}) != 1:
        raise ValueError("batch_page_tables requires matching block sizes")
    if not any(c.valid > 0 for c in caches):
        raise ValueError("batch_page_tables requires at least one non-empty cache")
    if any(c.pool.key_blocks is None for c in caches):
        raise ValueError("batch_page_tables requires allocated block storage")
    index_dtype = index_dtype or torch.long
    block_size = caches[0].block_size
    max_blocks = max(max(len(c.block_table) for c in caches), 1)
    max_len = max(c.valid for c in caches)
    # one pinned staging buffer: column 0 the row's length, then its padded table
    device = caches[0].pool.key_blocks.device
    host = torch.full((len(caches), max_blocks + 1), -1, dtype=index_dtype, pin_memory=device.type == "cuda")
    for row, c in enumerate(caches):
        c.batched_page_table_calls += 1
        c.page_table_entries_total += len(c.block_table)
        c.page_table_tensor_calls += 1
        host[row, 0] = c.valid
        if c.block_table:
            host[row, 1:1 + len(c.block_table)] = torch.tensor(c.block_table, dtype=index_dtype)
    staged = host.to(device, non_blocking=True)
    tables, lengths = staged[:, 1:], staged[:, 0].contiguous()
    mask = torch.arange(max_len, device=device)[None, :] < lengths[:, None]
    return BatchedFullAttentionPageTables(tables, lengths, mask, block_size, max_blocks, max_len,
                                          tuple(c.pool.key_blocks for c in caches),
                                          tuple(c.pool.value_blocks for c in caches))


def batch_kv_tensors(caches: Sequence[FullAttentionCache]) -> tuple[Any, Any, Any]:
    """Dense zero-padded (B, kv_heads, max_valid, head_dim) K, V and the (B, max_valid) valid mask
    (src/decode_state.py:501-542 semantics), gathered on the device: one kv_gather over a shared pool,
    else one per request."""
    import torch

    meta = batch_page_tables(caches)
    for c in caches:
        c.gather_view_calls += 1
        c.gather_copied_tokens += c.valid
    pool = meta.key_blocks[0]
    if all(k is pool for k in meta.key_blocks):
        keys, values = ops.kv_gather(pool, meta.value_blocks[0], meta.block_tables, meta.sequence_lengths,
                                     meta.max_sequence_length)
        return keys, values, meta.valid_mask
    shape = (len(caches), pool.shape[1], meta.max_sequence_length, pool.shape[3])
    keys = torch.zeros(shape, dtype=pool.dtype, device=pool.device)
    values = torch.zeros_like(keys)
    for row, c in enumerate(caches):
        if c.valid:
            k, v = ops.kv_gather(c.pool.key_blocks, c.pool.value_blocks, meta.block_tables[row:row + 1],
                                 meta.sequence_lengths[row:row + 1], c.valid)
            keys[row, :, :c.valid] = k[0]
            values[row, :, :c.valid] = v[0]
    return keys, values, meta.valid_mask
